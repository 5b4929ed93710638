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
#include "common.cuh"
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

// cp.async of a [64 token][d] slice (rows t < valid, channels < D, zero elsewhere) into a tile
__device__ __forceinline__ void load_tokens(uint8_t* tile, const bf16* __restrict__ src,
                                            int64_t row0, int64_t row_stride, int valid, int D) {
  const uint32_t base = smem_u32(tile);
  for (int q = threadIdx.x; q < C * (DP / 8); q += NT) {
    const int r = q >> 4, j = q & 15;
    const bool ok = r < valid && 8 * j < D;
    const bf16* p = ok ? src + (row0 + r) * row_stride + 8 * j : src;
    cp_async16(base + sw_chunk(64, r, j), p, ok ? 16u : 0u);
  }
}

__device__ __forceinline__ void load_linear(uint8_t* dst, const uint8_t* __restrict__ src, uint32_t bytes) {
  const uint32_t base = smem_u32(dst);
  for (uint32_t q = threadIdx.x; q < bytes / 16; q += NT) cp_async16(base + 16 * q, src + 16 * q, 16u);
}

__device__ __forceinline__ void store_linear(uint8_t* __restrict__ dst, const uint8_t* src, uint32_t bytes) {
  for (uint32_t q = threadIdx.x; q < bytes / 16; q += NT)
    reinterpret_cast<uint4*>(dst)[q] = reinterpret_cast<const uint4*>(src)[q];
}

__device__ __forceinline__ void load_beta(float* bsm, const bf16* __restrict__ beta, int64_t row0,
                                          int H, int valid) {
  if (threadIdx.x < C) {
    const int t = threadIdx.x;
    bsm[t] = t < valid ? __bfloat162float(beta[(row0 + t) * H]) : 0.f;
  }
}

// T'[t][s] = X[t][s] * beta_s (bf16 tile images, one 8-element chunk per step)
__device__ __forceinline__ void scale_columns(uint8_t* Tt, const uint8_t* Xt, const float* bsm) {
  for (int q = threadIdx.x; q < 64 * 8; q += NT) {
    const int r = q >> 3, j = q & 7;
    const uint32_t off = sw_chunk(64, r, j);
    uint4 w = *reinterpret_cast<const uint4*>(Xt + off);
    bf16* e = reinterpret_cast<bf16*>(&w);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = __float2bfloat16_rn(__bfloat162float(e[i]) * bsm[8 * j + i]);
    *reinterpret_cast<uint4*>(Tt + off) = w;
  }
}

__device__ __forceinline__ void ld64(uint32_t tm, int col, float (&v)[64]) {
  float* a = v;
  tmem_ld32(tm + (uint32_t)col, *reinterpret_cast<float(*)[32]>(a));
  tmem_ld32(tm + (uint32_t)col + 32, *reinterpret_cast<float(*)[32]>(a + 32));
  tmem_wait_ld();
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

// ------------------------------------------------------------------------------------------
// prep: X = (I + strictly_lower(diag(beta) K K^T))^-1 per chunk, bf16 tile image [64 t][64 s]
// ------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(NT) scan_prep_kernel(const bf16* __restrict__ k,
                                                       const bf16* __restrict__ beta,
                                                       uint8_t* __restrict__ xt, int T, int H,
                                                       int D, int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* Kt = sm;                                   // 16 KB
  uint8_t* Xs = sm + TILE_TD;                         // 8 KB
  float* A = reinterpret_cast<float*>(sm + TILE_TD + TILE_TT);  // [64][65]
  __shared__ float bsm[C];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC, b = bh / H, h = bh % H;
  const int t0 = c * C, valid = min(C, T - t0);
  const int64_t row0 = (int64_t)b * T + t0;
  load_tokens(Kt, k + (int64_t)h * D, row0, (int64_t)H * D, valid, D);
  cp_async_commit();
  load_beta(bsm, beta + h, row0, H, valid);
  if (tid == 0) { mbar_init(&bar, 1); mbar_fence_init(); }
  if (warp == 0) { tmem_alloc(&tbase, 64); tmem_relinquish(); }
  cp_async_wait_all();
  publish();
  const uint32_t tm = tbase;
  if (tid == 0) {
    const uint32_t id = idesc_bf16(64, 64, 0, 0);
    for (int s = 0; s < DP / 16; ++s)
      umma_bf16(tm, desc_k(smem_u32(Kt), 64, s), desc_k(smem_u32(Kt), 64, s), id, s > 0 ? 1u : 0u);
    umma_commit(&bar);
  }
  uint32_t phase = 0;
  const bool ok = mma_wait(&bar, phase, status);
  const int row = warp * 16 + (lane & 15);
  float v[64];
  ld64(taddr(tm, warp * 32, 0), 0, v);
  if (lane < 16) {
#pragma unroll
    for (int s = 0; s < 64; ++s) A[row * 65 + s] = s < row ? bsm[row] * v[s] : 0.f;
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
  store_linear(xt + (size_t)blockIdx.x * TILE_TT, Xs, TILE_TT);
}

// ------------------------------------------------------------------------------------------
// forward: one CTA per (b, h); thread j <-> tensor-memory lane j <-> value index j
// ------------------------------------------------------------------------------------------
struct FwdSmem {
  static constexpr uint32_t Kt = 0, Qt = Kt + TILE_TD, Vt = Qt + TILE_TD, Xt = Vt + TILE_TD,
                            Tt = Xt + TILE_TT, Pt = Tt + TILE_TT, Wr = Pt + TILE_TT,
                            Ha = Wr + TILE_JT, Da = Ha + TILE_JI, END = Da + TILE_JT;
};
// tensor-memory columns
constexpr int F_H = 0, F_U = 128, F_W = 192, F_X = 256, F_QK = 320, F_O = 384;

__global__ void __launch_bounds__(NT, 1) scan_fwd_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
    const bf16* __restrict__ beta, const float* __restrict__ s0, const uint8_t* __restrict__ xt,
    bf16* __restrict__ o, float* __restrict__ sn, uint8_t* __restrict__ hck, int T, int H, int D,
    int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Kt = sm + FwdSmem::Kt, *Qt = sm + FwdSmem::Qt, *Vt = sm + FwdSmem::Vt;
  uint8_t *Xt = sm + FwdSmem::Xt, *Tt = sm + FwdSmem::Tt, *Pt = sm + FwdSmem::Pt;
  uint8_t *Wr = sm + FwdSmem::Wr, *Ha = sm + FwdSmem::Ha, *Da = sm + FwdSmem::Da;
  __shared__ float bsm[C];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int64_t ld = (int64_t)H * D;  // elements between consecutive tokens of one head
  if (tid == 0) { mbar_init(&bar, 1); mbar_fence_init(); }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, warp * 32, 0);  // this warp's lane quarter
  // H^T row j = column j of the initial state
  {
    const int j = tid;
    float row[DP];
#pragma unroll
    for (int i = 0; i < DP; ++i) row[i] = (i < D && j < D) ? s0[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) tmem_st32(lane_tm + F_H + 32 * q4, *reinterpret_cast<float(*)[32]>(row + 32 * q4));
    tmem_wait_st();
    st_row64_bf16(Ha, 128, j, 0, row);
    st_row64_bf16(Ha, 128, j, 1, row + 64);
  }
  publish();
  uint32_t phase = 0;
  bool ok = true;
  const uint32_t sK = smem_u32(Kt), sQ = smem_u32(Qt), sV = smem_u32(Vt), sT = smem_u32(Tt);
  const uint32_t sP = smem_u32(Pt), sW = smem_u32(Wr), sH = smem_u32(Ha), sD = smem_u32(Da);
  for (int c = 0; c < NC && ok; ++c) {
    const int t0 = c * C, valid = min(C, T - t0);
    const int64_t row0 = (int64_t)b * T + t0;
    load_tokens(Kt, k + (int64_t)h * D, row0, ld, valid, D);
    load_tokens(Qt, q + (int64_t)h * D, row0, ld, valid, D);
    load_tokens(Vt, v + (int64_t)h * D, row0, ld, valid, D);
    load_linear(Xt, xt + ((size_t)bh * NC + c) * TILE_TT, TILE_TT);
    cp_async_commit();
    load_beta(bsm, beta + h, row0, H, valid);
    // checkpoint H_c (the bf16 copy the chunk's products read) while the loads land
    store_linear(hck + ((size_t)bh * NC + c) * TILE_JI, Ha, TILE_JI);
    cp_async_wait_all();
    __syncthreads();
    scale_columns(Tt, Xt, bsm);
    publish();
    if (tid == 0) {
      const uint32_t id_tn = idesc_bf16(128, 64, 1, 0);  // A MN-major, B K-major
      for (int s = 0; s < 4; ++s) {
        umma_bf16(tm + F_U, desc_mn(sV, 64, s), desc_k(sT, 64, s), id_tn, s > 0);
        umma_bf16(tm + F_W, desc_mn(sK, 64, s), desc_k(sT, 64, s), id_tn, s > 0);
      }
      const uint32_t id_qk = idesc_bf16(64, 64, 0, 0);
      for (int s = 0; s < 8; ++s) umma_bf16(tm + F_QK, desc_k(sQ, 64, s), desc_k(sK, 64, s), id_qk, s > 0);
      umma_commit(&bar);
    }
    ok = mma_wait(&bar, phase, status);
    {
      float w[64];
      ld64(lane_tm, F_W, w);
      st_row64_bf16(Wr, 128, tid, 0, w);  // W^T row i: MN-major B operand [i][t]
      float p[64];
      ld64(lane_tm, F_QK, p);
      const int t = warp * 16 + (lane & 15);
      if (lane < 16) {
#pragma unroll
        for (int s = 0; s < 64; ++s) p[s] = s <= t ? p[s] : 0.f;
        st_row64_bf16(Pt, 64, t, 0, p);
      }
    }
    publish();
    if (tid == 0) {
      const uint32_t id_hw = idesc_bf16(128, 64, 0, 1);  // A K-major (H^T), B MN-major (W^T rows)
      for (int s = 0; s < 8; ++s) umma_bf16(tm + F_X, desc_k(sH, 128, s), desc_mn(sW, 128, s), id_hw, s > 0);
      const uint32_t id_qh = idesc_bf16(64, 128, 0, 0);  // O = Q H: both K-major
      for (int s = 0; s < 8; ++s) umma_bf16(tm + F_O, desc_k(sQ, 64, s), desc_k(sH, 128, s), id_qh, s > 0);
      umma_commit(&bar);
    }
    ok = ok && mma_wait(&bar, phase, status);
    {
      float u[64], x[64];
      ld64(lane_tm, F_U, u);
      ld64(lane_tm, F_X, x);
#pragma unroll
      for (int s = 0; s < 64; ++s) u[s] -= x[s];
      st_row64_bf16(Da, 128, tid, 0, u);  // delta^T row j: [j][t]
    }
    publish();
    if (tid == 0) {
      const uint32_t id_dk = idesc_bf16(128, 128, 0, 1);  // H^T += delta^T K (B MN-major)
      for (int s = 0; s < 4; ++s) umma_bf16(tm + F_H, desc_k(sD, 128, s), desc_mn(sK, 64, s), id_dk, 1u);
      const uint32_t id_pd = idesc_bf16(64, 128, 0, 0);  // O += P delta
      for (int s = 0; s < 4; ++s) umma_bf16(tm + F_O, desc_k(sP, 64, s), desc_k(sD, 128, s), id_pd, 1u);
      umma_commit(&bar);
    }
    ok = ok && mma_wait(&bar, phase, status);
    {
      // O rows: lanes 0-15 of each warp hold tokens t = 16 w + l
      const int t = warp * 16 + (lane & 15);
      float orow[DP];
      ld64(lane_tm, F_O, *reinterpret_cast<float(*)[64]>(orow));
      ld64(lane_tm, F_O + 64, *reinterpret_cast<float(*)[64]>(orow + 64));
      if (lane < 16 && t < valid) {
        bf16* dst = o + (row0 + t) * ld + (int64_t)h * D;
        for (int i = 0; i < D; i += 8) {
          uint4 w;
          w.x = pack_bf16(orow[i], orow[i + 1]);
          w.y = pack_bf16(orow[i + 2], orow[i + 3]);
          w.z = pack_bf16(orow[i + 4], orow[i + 5]);
          w.w = pack_bf16(orow[i + 6], orow[i + 7]);
          *reinterpret_cast<uint4*>(dst + i) = w;
        }
      }
      float hrow[DP];
      ld64(lane_tm, F_H, *reinterpret_cast<float(*)[64]>(hrow));
      ld64(lane_tm, F_H + 64, *reinterpret_cast<float(*)[64]>(hrow + 64));
      st_row64_bf16(Ha, 128, tid, 0, hrow);
      st_row64_bf16(Ha, 128, tid, 1, hrow + 64);
      if (c == NC - 1) {
        const int j = tid;
        if (j < D)
          for (int i = 0; i < D; ++i) sn[(int64_t)bh * D * D + (int64_t)i * D + j] = hrow[i];
      }
    }
    publish();
  }
  if (NC == 0) {
    const int j = tid;
    if (j < D)
      for (int i = 0; i < D; ++i) sn[(int64_t)bh * D * D + (int64_t)i * D + j] = s0[(int64_t)bh * D * D + (int64_t)i * D + j];
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tm, 512);
}

// ------------------------------------------------------------------------------------------
// backward, sequential: dH^T chain in tensor memory; checkpoints dH_{c+1} per chunk
// ------------------------------------------------------------------------------------------
struct DhSmem {
  static constexpr uint32_t Kt = 0, Qt = Kt + TILE_TD, Gt = Qt + TILE_TD, Xt = Gt + TILE_TD,
                            Tt = Xt + TILE_TT, Pt = Tt + TILE_TT, Wk = Pt + TILE_TT,
                            Ha = Wk + TILE_JT, Da = Ha + TILE_JI, END = Da + TILE_JT;
};
constexpr int G_H = 0, G_W = 128, G_D = 192, G_QK = 256;

__global__ void __launch_bounds__(NT, 1) scan_dh_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ beta,
    const uint8_t* __restrict__ xt, const bf16* __restrict__ dout, const float* __restrict__ dsn,
    float* __restrict__ ds0, uint8_t* __restrict__ dhck, int T, int H, int D, int NC, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Kt = sm + DhSmem::Kt, *Qt = sm + DhSmem::Qt, *Gt = sm + DhSmem::Gt;
  uint8_t *Xt = sm + DhSmem::Xt, *Tt = sm + DhSmem::Tt, *Pt = sm + DhSmem::Pt;
  uint8_t *Wk = sm + DhSmem::Wk, *Ha = sm + DhSmem::Ha, *Da = sm + DhSmem::Da;
  __shared__ float bsm[C];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int64_t ld = (int64_t)H * D;
  if (tid == 0) { mbar_init(&bar, 1); mbar_fence_init(); }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, warp * 32, 0);
  {
    const int j = tid;
    float row[DP];
#pragma unroll
    for (int i = 0; i < DP; ++i)
      row[i] = (dsn != nullptr && i < D && j < D) ? dsn[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) tmem_st32(lane_tm + G_H + 32 * q4, *reinterpret_cast<float(*)[32]>(row + 32 * q4));
    tmem_wait_st();
    st_row64_bf16(Ha, 128, j, 0, row);
    st_row64_bf16(Ha, 128, j, 1, row + 64);
  }
  publish();
  uint32_t phase = 0;
  bool ok = true;
  const uint32_t sK = smem_u32(Kt), sQ = smem_u32(Qt), sG = smem_u32(Gt), sT = smem_u32(Tt);
  const uint32_t sP = smem_u32(Pt), sW = smem_u32(Wk), sH = smem_u32(Ha), sD = smem_u32(Da);
  for (int c = NC - 1; c >= 0 && ok; --c) {
    const int t0 = c * C, valid = min(C, T - t0);
    const int64_t row0 = (int64_t)b * T + t0;
    load_tokens(Kt, k + (int64_t)h * D, row0, ld, valid, D);
    load_tokens(Qt, q + (int64_t)h * D, row0, ld, valid, D);
    load_tokens(Gt, dout + (int64_t)h * D, row0, ld, valid, D);
    load_linear(Xt, xt + ((size_t)bh * NC + c) * TILE_TT, TILE_TT);
    cp_async_commit();
    load_beta(bsm, beta + h, row0, H, valid);
    store_linear(dhck + ((size_t)bh * NC + c) * TILE_JI, Ha, TILE_JI);  // dH_{c+1}
    cp_async_wait_all();
    __syncthreads();
    scale_columns(Tt, Xt, bsm);
    publish();
    if (tid == 0) {
      const uint32_t id_tn = idesc_bf16(128, 64, 1, 0);
      for (int s = 0; s < 4; ++s) umma_bf16(tm + G_W, desc_mn(sK, 64, s), desc_k(sT, 64, s), id_tn, s > 0);
      const uint32_t id_qk = idesc_bf16(64, 64, 0, 0);
      for (int s = 0; s < 8; ++s) umma_bf16(tm + G_QK, desc_k(sQ, 64, s), desc_k(sK, 64, s), id_qk, s > 0);
      // ddelta^T = dH^T K^T (+ dO^T P below)
      const uint32_t id_hk = idesc_bf16(128, 64, 0, 0);
      for (int s = 0; s < 8; ++s) umma_bf16(tm + G_D, desc_k(sH, 128, s), desc_k(sK, 64, s), id_hk, s > 0);
      // dH^T += dO^T Q
      const uint32_t id_oq = idesc_bf16(128, 128, 1, 1);
      for (int s = 0; s < 4; ++s) umma_bf16(tm + G_H, desc_mn(sG, 64, s), desc_mn(sQ, 64, s), id_oq, 1u);
      umma_commit(&bar);
    }
    ok = mma_wait(&bar, phase, status);
    {
      float w[64];
      ld64(lane_tm, G_W, w);
      st_row64_bf16(Wk, 128, tid, 0, w);  // W^T row i: K-major B [i][t]
      float p[64];
      ld64(lane_tm, G_QK, p);
      const int t = warp * 16 + (lane & 15);
      if (lane < 16) {
#pragma unroll
        for (int s = 0; s < 64; ++s) p[s] = s <= t ? p[s] : 0.f;
        st_row64_bf16(Pt, 64, t, 0, p);
      }
    }
    publish();
    if (tid == 0) {
      const uint32_t id_op = idesc_bf16(128, 64, 1, 1);  // dO^T (MN) x P (MN)
      for (int s = 0; s < 4; ++s) umma_bf16(tm + G_D, desc_mn(sG, 64, s), desc_mn(sP, 64, s), id_op, 1u);
      umma_commit(&bar);
    }
    ok = ok && mma_wait(&bar, phase, status);
    {
      float d[64];
      ld64(lane_tm, G_D, d);
      st_row64_bf16(Da, 128, tid, 0, d);  // ddelta^T row j
    }
    publish();
    if (tid == 0) {
      const uint32_t id_dw = idesc_bf16(128, 128, 0, 0, 1);  // dH^T -= ddelta^T W
      for (int s = 0; s < 4; ++s) umma_bf16(tm + G_H, desc_k(sD, 128, s), desc_k(sW, 128, s), id_dw, 1u);
      umma_commit(&bar);
    }
    ok = ok && mma_wait(&bar, phase, status);
    {
      float hrow[DP];
      ld64(lane_tm, G_H, *reinterpret_cast<float(*)[64]>(hrow));
      ld64(lane_tm, G_H + 64, *reinterpret_cast<float(*)[64]>(hrow + 64));
      st_row64_bf16(Ha, 128, tid, 0, hrow);
      st_row64_bf16(Ha, 128, tid, 1, hrow + 64);
      if (c == 0) {
        const int j = tid;
        if (j < D)
          for (int i = 0; i < D; ++i) ds0[(int64_t)bh * D * D + (int64_t)i * D + j] = hrow[i];
      }
    }
    publish();
  }
  if (NC == 0) {
    const int j = tid;
    if (j < D)
      for (int i = 0; i < D; ++i)
        ds0[(int64_t)bh * D * D + (int64_t)i * D + j] = dsn ? dsn[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
  }
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
constexpr int R_KK = 0, R_QK = 64, R_W = 128, R_U = 192, R_DD = 256, R_X = 320;   // batches 1-2
constexpr int R_DP = 64, R_DW = 128, R_DV = 256, R_DT = 384;                      // batch 3
constexpr int R_DQ = 128, R_Y = 256, R_Z = 320, R_DK = 128;                       // batches 4-7

__global__ void __launch_bounds__(NT, 1) scan_grad_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
    const bf16* __restrict__ beta, const uint8_t* __restrict__ xt, const uint8_t* __restrict__ hck,
    const uint8_t* __restrict__ dhck, const bf16* __restrict__ dout, bf16* __restrict__ dq,
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
  __shared__ float bsm[C], db1[C];
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int c = blockIdx.x % NC, bh = blockIdx.x / NC, b = bh / H, h = bh % H;
  const int t0 = c * C, valid = min(C, T - t0);
  const int64_t ld = (int64_t)H * D;
  const int64_t row0 = (int64_t)b * T + t0;
  const int trow = warp * 16 + (lane & 15);  // token row of an M=64 accumulator (lane < 16)
  const bool rowlane = lane < 16;
  load_tokens(Qt, q + (int64_t)h * D, row0, ld, valid, D);
  load_tokens(Kt, k + (int64_t)h * D, row0, ld, valid, D);
  load_tokens(Vt, v + (int64_t)h * D, row0, ld, valid, D);
  load_tokens(Gt, dout + (int64_t)h * D, row0, ld, valid, D);
  const size_t chunk = (size_t)bh * NC + c;
  load_linear(Ht, hck + chunk * TILE_JI, TILE_JI);
  load_linear(dHt, dhck + chunk * TILE_JI, TILE_JI);
  load_linear(Xt, xt + chunk * TILE_TT, TILE_TT);
  cp_async_commit();
  load_beta(bsm, beta + h, row0, H, valid);
  if (tid == 0) { mbar_init(&bar, 1); mbar_fence_init(); }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  cp_async_wait_all();
  __syncthreads();
  scale_columns(Tt, Xt, bsm);
  publish();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, warp * 32, 0);
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
    for (int s = 0; s < 8; ++s) {
      umma_bf16(tm + R_KK, desc_k(sK, 64, s), desc_k(sK, 64, s), id64, s > 0);
      umma_bf16(tm + R_QK, desc_k(sQ, 64, s), desc_k(sK, 64, s), id64, s > 0);
    }
    const uint32_t id_tn = idesc_bf16(128, 64, 1, 0);
    for (int s = 0; s < 4; ++s) {
      umma_bf16(tm + R_W, desc_mn(sK, 64, s), desc_k(sT, 64, s), id_tn, s > 0);
      umma_bf16(tm + R_U, desc_mn(sV, 64, s), desc_k(sT, 64, s), id_tn, s > 0);
    }
    const uint32_t id_hk = idesc_bf16(128, 64, 0, 0);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DD, desc_k(sdH, 128, s), desc_k(sK, 64, s), id_hk, s > 0);
    umma_commit(&bar);
  }
  ok = mma_wait(&bar, phase, status);
  {
    float w[64];
    ld64(lane_tm, R_W, w);
    st_row64_bf16(Wr, 128, tid, 0, w);
    float p[64];
    ld64(lane_tm, R_QK, p);
    if (rowlane) {
#pragma unroll
      for (int s = 0; s < 64; ++s) p[s] = s <= trow ? p[s] : 0.f;
      st_row64_bf16(Pt, 64, trow, 0, p);
    }
  }
  publish();
  // batch 2: X = H^T W^T; ddelta^T += dO^T P
  if (tid == 0 && ok) {
    const uint32_t id_hw = idesc_bf16(128, 64, 0, 1);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_X, desc_k(sH, 128, s), desc_mn(sW, 128, s), id_hw, s > 0);
    const uint32_t id_op = idesc_bf16(128, 64, 1, 1);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_DD, desc_mn(sG, 64, s), desc_mn(sP, 64, s), id_op, 1u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float u[64], x[64];
    ld64(lane_tm, R_U, u);
    ld64(lane_tm, R_X, x);
#pragma unroll
    for (int s = 0; s < 64; ++s) u[s] -= x[s];
    st_row64_bf16(Dt, 128, tid, 0, u);  // delta^T [j][t]
    float d[64];
    ld64(lane_tm, R_DD, d);
    st_row64_bf16(dDt, 128, tid, 0, d);  // ddelta^T [j][t]
  }
  publish();
  // batch 3: dP = dO delta^T; dW = -ddelta H^T; dV = T'^T ddelta; dT' = ddelta V^T
  if (tid == 0 && ok) {
    const uint32_t id_dp = idesc_bf16(64, 64, 0, 1);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DP, desc_k(sG, 64, s), desc_mn(sD, 128, s), id_dp, s > 0);
    const uint32_t id_dw = idesc_bf16(64, 128, 1, 1, 1);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DW, desc_mn(sdD, 128, s), desc_mn(sH, 128, s), id_dw, s > 0);
    const uint32_t id_dv = idesc_bf16(64, 128, 1, 0);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_DV, desc_mn(sT, 64, s), desc_k(sdD, 128, s), id_dv, s > 0);
    const uint32_t id_dt = idesc_bf16(64, 64, 1, 0);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DT, desc_mn(sdD, 128, s), desc_k(sV, 64, s), id_dt, s > 0);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float a[64];
    ld64(lane_tm, R_DP, a);
    if (rowlane) {
#pragma unroll
      for (int s = 0; s < 64; ++s) a[s] = s <= trow ? a[s] : 0.f;
      st_row64_bf16(dPt, 64, trow, 0, a);
    }
    float r[DP];
    ld64(lane_tm, R_DW, *reinterpret_cast<float(*)[64]>(r));
    ld64(lane_tm, R_DW + 64, *reinterpret_cast<float(*)[64]>(r + 64));
    if (rowlane) {
      st_row64_bf16(dWt, 64, trow, 0, r);
      st_row64_bf16(dWt, 64, trow, 1, r + 64);
    }
    ld64(lane_tm, R_DV, *reinterpret_cast<float(*)[64]>(r));
    ld64(lane_tm, R_DV + 64, *reinterpret_cast<float(*)[64]>(r + 64));
    if (rowlane && trow < valid) {
      bf16* dst = dv + (row0 + trow) * ld + (int64_t)h * D;
      for (int i = 0; i < D; i += 8) {
        uint4 w4;
        w4.x = pack_bf16(r[i], r[i + 1]); w4.y = pack_bf16(r[i + 2], r[i + 3]);
        w4.z = pack_bf16(r[i + 4], r[i + 5]); w4.w = pack_bf16(r[i + 6], r[i + 7]);
        *reinterpret_cast<uint4*>(dst + i) = w4;
      }
    }
  }
  publish();
  // batch 4: dQ = dO H^T + dP K; dT' += dW K^T
  if (tid == 0 && ok) {
    const uint32_t id_oh = idesc_bf16(64, 128, 0, 1);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DQ, desc_k(sG, 64, s), desc_mn(sH, 128, s), id_oh, s > 0);
    const uint32_t id_pk = idesc_bf16(64, 128, 0, 1);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_DQ, desc_k(sdP, 64, s), desc_mn(sK, 64, s), id_pk, 1u);
    const uint32_t id_wk = idesc_bf16(64, 64, 0, 0);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DT, desc_k(sdW, 64, s), desc_k(sK, 64, s), id_wk, 1u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float r[DP];
    ld64(lane_tm, R_DQ, *reinterpret_cast<float(*)[64]>(r));
    ld64(lane_tm, R_DQ + 64, *reinterpret_cast<float(*)[64]>(r + 64));
    if (rowlane && trow < valid) {
      bf16* dst = dq + (row0 + trow) * ld + (int64_t)h * D;
      for (int i = 0; i < D; i += 8) {
        uint4 w4;
        w4.x = pack_bf16(r[i], r[i + 1]); w4.y = pack_bf16(r[i + 2], r[i + 3]);
        w4.z = pack_bf16(r[i + 4], r[i + 5]); w4.w = pack_bf16(r[i + 6], r[i + 7]);
        *reinterpret_cast<uint4*>(dst + i) = w4;
      }
    }
    // dT' row t: dX = dT' diag(beta) (bf16 operand), dT' * X products for dbeta's first part
    float dt[64];
    ld64(lane_tm, R_DT, dt);
    if (rowlane) {
      float xr[64], dx[64];
#pragma unroll
      for (int s = 0; s < 64; ++s) {
        xr[s] = __bfloat162float(*reinterpret_cast<const bf16*>(Xt + sw_offset(64, trow, s)));
        dx[s] = dt[s] * bsm[s];
        scr[trow * 65 + s] = dt[s] * xr[s];
      }
      st_row64_bf16(dXt, 64, trow, 0, dx);
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
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_Y, desc_k(sdX, 64, s), desc_k(sX, 64, s), id, s > 0);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float y[64];
    ld64(lane_tm, R_Y, y);
    if (rowlane) st_row64_bf16(Yt, 64, trow, 0, y);
  }
  publish();
  // batch 6: Z = X^T Y; dA = -Z (strictly lower)
  if (tid == 0 && ok) {
    const uint32_t id = idesc_bf16(64, 64, 1, 1);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_Z, desc_mn(sX, 64, s), desc_mn(sY, 64, s), id, s > 0);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  float db2 = 0.f;
  {
    float z[64], kk[64];
    ld64(lane_tm, R_Z, z);
    ld64(lane_tm, R_KK, kk);
    if (rowlane) {
      const float bt = bsm[trow];
#pragma unroll
      for (int s = 0; s < 64; ++s) {
        const float da = s < trow ? -z[s] : 0.f;
        db2 = fmaf(da, kk[s], db2);
        scr[trow * 65 + s] = bt * da;  // dG
      }
    }
  }
  __syncthreads();
  if (rowlane) {
    float g[64];
#pragma unroll
    for (int s = 0; s < 64; ++s) g[s] = scr[trow * 65 + s] + scr[s * 65 + trow];
    st_row64_bf16(dGt, 64, trow, 0, g);
    if (trow < valid) dbeta[(row0 + trow) * H + h] = __float2bfloat16_rn(db1[trow] + db2);
  }
  publish();
  // batch 7: dK = dP^T Q + delta dH'^T + T'^T dW + (dG + dG^T) K
  if (tid == 0 && ok) {
    const uint32_t id_mn = idesc_bf16(64, 128, 1, 1);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_DK, desc_mn(sdP, 64, s), desc_mn(sQ, 64, s), id_mn, s > 0);
    for (int s = 0; s < 8; ++s) umma_bf16(tm + R_DK, desc_mn(sD, 128, s), desc_mn(sdH, 128, s), id_mn, 1u);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_DK, desc_mn(sT, 64, s), desc_mn(sdW, 64, s), id_mn, 1u);
    const uint32_t id_gk = idesc_bf16(64, 128, 0, 1);
    for (int s = 0; s < 4; ++s) umma_bf16(tm + R_DK, desc_k(sdG, 64, s), desc_mn(sK, 64, s), id_gk, 1u);
    umma_commit(&bar);
  }
  ok = ok && mma_wait(&bar, phase, status);
  {
    float r[DP];
    ld64(lane_tm, R_DK, *reinterpret_cast<float(*)[64]>(r));
    ld64(lane_tm, R_DK + 64, *reinterpret_cast<float(*)[64]>(r + 64));
    if (rowlane && trow < valid) {
      bf16* dst = dk + (row0 + trow) * ld + (int64_t)h * D;
      for (int i = 0; i < D; i += 8) {
        uint4 w4;
        w4.x = pack_bf16(r[i], r[i + 1]); w4.y = pack_bf16(r[i + 2], r[i + 3]);
        w4.z = pack_bf16(r[i + 4], r[i + 5]); w4.w = pack_bf16(r[i + 6], r[i + 7]);
        *reinterpret_cast<uint4*>(dst + i) = w4;
      }
    }
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
  const size_t n = seqs * nc * (TILE_TT + TILE_JI);
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
  uint8_t* hck = xt + (size_t)B * H * NC * TILE_TT;
  if (NC > 0) {
    const size_t sp = smem_bytes(TILE_TD + TILE_TT + 64 * 65 * 4);
    VB_CUDA_CHECK(cudaFuncSetAttribute(scan_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sp), "prep attr");
    scan_prep_kernel<<<B * H * NC, NT, sp, st>>>((const bf16*)k, (const bf16*)beta, xt, T, H, D, NC, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 prep");
  }
  const size_t sf = smem_bytes(FwdSmem::END);
  VB_CUDA_CHECK(cudaFuncSetAttribute(scan_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sf), "fwd attr");
  scan_fwd_kernel<<<B * H, NT, sf, st>>>((const bf16*)q, (const bf16*)k, (const bf16*)v, (const bf16*)beta,
                                         state0, xt, (bf16*)o, state_n, hck, T, H, D, NC, status);
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
  const uint8_t* hck = xt + (size_t)B * H * NC * TILE_TT;
  uint8_t* dhck = (uint8_t*)workspace;
  const size_t sd = smem_bytes(DhSmem::END);
  VB_CUDA_CHECK(cudaFuncSetAttribute(scan_dh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sd), "dh attr");
  scan_dh_kernel<<<B * H, NT, sd, st>>>((const bf16*)q, (const bf16*)k, (const bf16*)beta, xt, (const bf16*)dout,
                                        dstate_n, dstate0, dhck, T, H, D, NC, status);
  VB_LAUNCH_CHECK("delta_scan_bf16 dh");
  if (NC > 0) {
    const size_t sg = smem_bytes(GrSmem::END);
    VB_CUDA_CHECK(cudaFuncSetAttribute(scan_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sg), "grad attr");
    scan_grad_kernel<<<B * H * NC, NT, sg, st>>>((const bf16*)q, (const bf16*)k, (const bf16*)v, (const bf16*)beta,
                                                 xt, hck, dhck, (const bf16*)dout, (bf16*)dq, (bf16*)dk, (bf16*)dv,
                                                 (bf16*)dbeta, T, H, D, NC, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 grad");
  }
  return VB_OK;
}
