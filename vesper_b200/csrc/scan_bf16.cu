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
//   forward  two CTAs per sequence (one per half of the value index j) walk its chunks; H^T
//            lives in tensor memory (fp32, rows = value index j, columns = key index i). The bf16
//            copy of H_c that fed the chunk's products is checkpointed (the backward reuses it, no
//            recomputation of the chain).
//   backward two CTAs per sequence walk the chunks in reverse for the state gradient,
//            checkpointing the bf16 dH_{c+1}; then one persistent CTA per SM forms every local
//            gradient of a chunk from (H_c, dH_{c+1}) in five product stages: dq, dk, dv, dbeta.
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

// the additive shift of this thread's token (threads < 64) for the write-strength logits, or 0
__device__ __forceinline__ float fetch_shift(const float* __restrict__ shift, int64_t row0, int valid) {
  const int t = threadIdx.x;
  return (shift != nullptr && t < C && t < valid) ? shift[row0 + t] : 0.f;
}

// The write strength the scan uses: `raw` itself, or with `logit` set the reference's
// write_strength, beta = sigmoid(raw + shift) rounded to bf16 as torch.sigmoid's bf16 output is
// (1 / (1 + exp(-x)) in float32, vesper/recurrence.py:34-88).
__device__ __forceinline__ float beta_value(bf16 raw, int logit, float shift) {
  if (!logit) return __bfloat162float(raw);
  const float x = __bfloat162float(raw) + shift;
  return __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-x))));
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
  // Vt: V, then U; AF: float32 A [64][AS], then atom 0 of M; Ws: the X image, then W, then atom 1
  // of M; TT: [T'; T'] (128 rows x 64); Ps: P. During the solve Ws and TT hold the float32 X
  // [64][68] and the block products (3 x [16][20]).
  static constexpr uint32_t KQ = 0, Vt = TILE_JI, AF = Vt + TILE_TD, Ws = AF + 17 * 1024, TT = Ws + TILE_TD,
                            Ps = TT + TILE_JT, END = Ps + TILE_TT;
};
constexpr int NP = 256;

// X = (I + A)^-1 for the strictly lower A (float32 [64][AS]) into X (float32 [64][68]), 256
// threads, by blocks of 16 in three levels:
//   1. the four diagonal blocks X_II by forward substitution (a thread per column; the entries
//      above a block's diagonal come out as zeros);
//   2. the blocks below them inside each 32 x 32 half: X_10 = -X_11 (A_10 X_00) and
//      X_32 = -X_33 (A_32 X_22) (the two halves at once, a thread per 1 x 4 strip);
//   3. the lower-left 32 x 32 block: X[32:, :32] = -X[32:, 32:] (A[32:, :32] X[:32, :32]), every
//      thread a 1 x 4 strip of each product, the sums running over the blocks that are not zero.
// Five barriers instead of seven, and each product's dependent chain is at most 32 terms with four
// independent accumulators per thread. Entries above the diagonal blocks are not written.
// acc += a * v over the four lanes of a float4, two lanes per packed f32x2 FMA (each lane rounds
// as fmaf: the same results as four scalar FMAs)
__device__ __forceinline__ void fma4(float4& acc, float a, const float4& v) {
  const float2 lo = __ffma2_rn(make_float2(a, a), make_float2(v.x, v.y), make_float2(acc.x, acc.y));
  const float2 hi = __ffma2_rn(make_float2(a, a), make_float2(v.z, v.w), make_float2(acc.z, acc.w));
  acc = make_float4(lo.x, lo.y, hi.x, hi.y);
}

constexpr int XS = 68;  // row stride of X (16-byte aligned rows)
constexpr int AS = 68;  // row stride of A (16-byte aligned rows: written as 16-byte vectors)
constexpr int TS = 36;  // row stride of the products' scratch
__device__ __forceinline__ void invert_unit_lower(const float* A, float* X, float* Tm, int tid) {
  if (tid < C) {  // level 1
    const int o = 16 * (tid >> 4), j = tid & 15;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int s = 0; s < r; ++s) {
        if (s & 1) s1 = fmaf(A[(o + r) * AS + o + s], x[s], s1);
        else s0 = fmaf(A[(o + r) * AS + o + s], x[s], s0);
      }
      x[r] = (r == j ? 1.f : 0.f) - (s0 + s1);
      X[(o + r) * XS + o + j] = x[r];
    }
  }
  __syncthreads();
  // level 2: half hf (0: rows 16-31 x cols 0-15, 1: rows 48-63 x cols 32-47), row r, columns q4..q4+3
  const int hf = tid >> 6, r2 = (tid >> 2) & 15, q4 = 4 * (tid & 3);
  const bool l2 = tid < 128;
  if (l2) {  // T = A_(2hf+1, 2hf) X_(2hf, 2hf)
    const int ro = 32 * hf + 16, co = 32 * hf;
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      const float a = A[(ro + r2) * AS + co + s];
      const float4 x = *reinterpret_cast<const float4*>(X + (co + s) * XS + co + q4);
      fma4(t, a, x);
    }
    *reinterpret_cast<float4*>(Tm + (hf * 16 + r2) * TS + q4) = t;
  }
  __syncthreads();
  if (l2) {  // X_(2hf+1, 2hf) = -X_(2hf+1, 2hf+1) T
    const int ro = 32 * hf + 16, co = 32 * hf;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < 16; ++s) {
      const float a = X[(ro + r2) * XS + ro + s];
      const float4 t = *reinterpret_cast<const float4*>(Tm + (hf * 16 + s) * TS + q4);
      fma4(x, a, t);
    }
    *reinterpret_cast<float4*>(X + (ro + r2) * XS + co + q4) = make_float4(-x.x, -x.y, -x.z, -x.w);
  }
  __syncthreads();
  // level 3: row i of the lower 32 rows, columns j4..j4+3 of the left 32 columns
  const int i3 = tid >> 3, j4 = 4 * (tid & 7);
  {  // T = A[32:, :32] X[:32, :32]; X[k][j] is zero for k < 16 when j >= 16
    const int k0 = j4 >= 16 ? 16 : 0;
    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int k = k0; k < 32; ++k) {
      const float a = A[(32 + i3) * AS + k];
      const float4 x = *reinterpret_cast<const float4*>(X + k * XS + j4);
      fma4(t, a, x);
    }
    *reinterpret_cast<float4*>(Tm + i3 * TS + j4) = t;
  }
  __syncthreads();
  {  // X[32:, :32] = -X[32:, 32:] T; X[32 + i][32 + k] is zero for k >= 16 when i < 16
    const int k1 = i3 < 16 ? 16 : 32;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int k = 0; k < k1; ++k) {
      const float a = X[(32 + i3) * XS + 32 + k];
      const float4 t = *reinterpret_cast<const float4*>(Tm + k * TS + j4);
      fma4(x, a, t);
    }
    *reinterpret_cast<float4*>(X + (32 + i3) * XS + j4) = make_float4(-x.x, -x.y, -x.z, -x.w);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(NP, 2) scan_prep_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const bf16* __restrict__ beta, const float* __restrict__ shift,
    int logit, uint8_t* __restrict__ xt, int T, int H, int NC, int* status) {
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
  const float bsh = logit ? fetch_shift(shift, row0, valid) : 0.f;
  if (warp == 0) { tmem_alloc(&tbase, 256); tmem_relinquish(); }
  bool ok = mbar_wait(&lbar, 0);
  if (!ok) atomicOr(status, 4);
  if (tid < C) bsm[tid] = beta_value(bv, logit, bsh);  // after the tile wait: both loads in flight together
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
      const float bt = bsm[t];  // 0/1 masks and products below, not per-lane selects
#pragma unroll
      for (int e = 0; e < 32; e += 4)  // rows of AS floats: 16-byte aligned vectors
        *reinterpret_cast<float4*>(A + t * AS + c0 + e) =
            make_float4((c0 + e < t ? 1.f : 0.f) * (bt * v[e]), (c0 + e + 1 < t ? 1.f : 0.f) * (bt * v[e + 1]),
                        (c0 + e + 2 < t ? 1.f : 0.f) * (bt * v[e + 2]), (c0 + e + 3 < t ? 1.f : 0.f) * (bt * v[e + 3]));
    } else {
      const int t = lane128 - C;
#pragma unroll
      for (int e = 0; e < 32; ++e) v[e] *= c0 + e <= t ? 1.f : 0.f;
      st_row32_bf16(Ps, 64, t, c0, v);
    }
  }
  ok = publish_ok(ok);
  // 2. X (float32 over Ws and TT), then the bf16 X image into Ws and T' = bf16(X beta) into both
  //    halves of TT; every thread reads its 16 entries of X before any is overwritten
  {
    float* Xf = reinterpret_cast<float*>(Ws);
    invert_unit_lower(A, Xf, Xf + 64 * XS, tid);
    // each thread two 8-column chunks (row t, chunk c): 16-byte reads of X, 16-byte swizzled stores
    float xv[2][8];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int q = tid + NP * u, t = q >> 3, c = q & 7;
      const float4 a = *reinterpret_cast<const float4*>(Xf + t * XS + 8 * c);
      const float4 b = *reinterpret_cast<const float4*>(Xf + t * XS + 8 * c + 4);
      // loaded unconditionally (entries above the diagonal blocks are not written): a chunk lies
      // inside one 16-column block, so it is all zero or all kept
      // (a select, not a product: the unwritten entries may hold any bits)
      const bool keep = (c >> 1) <= (t >> 4);
      xv[u][0] = keep ? a.x : 0.f; xv[u][1] = keep ? a.y : 0.f; xv[u][2] = keep ? a.z : 0.f;
      xv[u][3] = keep ? a.w : 0.f; xv[u][4] = keep ? b.x : 0.f; xv[u][5] = keep ? b.y : 0.f;
      xv[u][6] = keep ? b.z : 0.f; xv[u][7] = keep ? b.w : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int q = tid + NP * u, t = q >> 3, c = q & 7;
      float xr[8], tr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        xr[i] = __bfloat162float(__float2bfloat16_rn(xv[u][i]));  // the bf16 X, and T' = bf16(X beta)
        tr[i] = xr[i] * bsm[8 * c + i];
      }
      uint4 xw, tw;
      xw.x = pack_bf16(xr[0], xr[1]); xw.y = pack_bf16(xr[2], xr[3]);
      xw.z = pack_bf16(xr[4], xr[5]); xw.w = pack_bf16(xr[6], xr[7]);
      tw.x = pack_bf16(tr[0], tr[1]); tw.y = pack_bf16(tr[2], tr[3]);
      tw.z = pack_bf16(tr[4], tr[5]); tw.w = pack_bf16(tr[6], tr[7]);
      *reinterpret_cast<uint4*>(Ws + sw_chunk(64, t, c)) = xw;
      *reinterpret_cast<uint4*>(TT + sw_chunk(128, t, c)) = tw;
      *reinterpret_cast<uint4*>(TT + sw_chunk(128, t + 64, c)) = tw;
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
// backward, chunk-parallel: every local gradient of one chunk from (H_c, dH_{c+1}).
// With R = V - K H_c (so delta = T' R), the chunk's gradients are five dependent product stages:
//   1  (K H)^T, ddelta^T = dH'^T K^T + dO^T P                         -> R^T = V^T - (K H)^T
//   2  delta^T = R^T T'^T, dW = -ddelta H^T, dV = T'^T ddelta, dT' = ddelta R^T
//   3  dP = dO delta^T (causal), Y = dX X^T (dX = dT' diag(beta)), dQ = dO H^T, dK = delta dH'^T
//   4  Z = X^T Y and Z^T = Y^T X, K K^T, dQ += dP K, dK += dP^T Q + T'^T dW
//   5  dK += dG K  (dG = diag(beta) dA symmetrised, dA = -Z strictly lower)
// dT' = dU V^T + dW K^T = ddelta (V - K H)^T needs no dW, and dV and dQ are read out while
// later stages run. One persistent CTA per SM walks chunks blockIdx.x, blockIdx.x + gridDim.x,
// ...: the next chunk's tiles stream into regions the current chunk has finished with, and its
// stage 1 runs while the current chunk's dQ and dK are read out. Regions (K and Q trade places
// between successive chunks of a CTA, so that the next K lands one stage early):
//   dH' 32 KB (read by stages 1, 3), H 32 KB (1-3), V 16 KB (stage 1 and its readout),
//   dO 16 KB (1, 3), P 8 KB (1)            -> the next chunk's after stages 1 and 3
//   Q 16 KB (4) -> next K after stage 4;  T' 8 KB (2, 4), X 8 KB (2-4) -> next after stage 4
//   K 16 KB (1, 4, 5) -> next Q after stage 5
// ------------------------------------------------------------------------------------------
struct GrSmem {
  static constexpr uint32_t DH = 0, HH = DH + TILE_JI, VV = HH + TILE_JI, GG = VV + TILE_TD, KA = GG + TILE_TD,
                            KB = KA + TILE_TD, PP = KB + TILE_TD, TT = PP + TILE_TT, XX = TT + TILE_TT,
                            Rt = XX + TILE_TT, dD = Rt + TILE_JT, Dt = dD + TILE_JT, Wd = Dt + TILE_JT,
                            END = Wd + TILE_TD;
  // reuse: R^T -> dX (+0) and dG (+8 KB); ddelta^T -> dV staging; delta^T -> dP (+0) and Y (+8 KB)
  // -> dK staging; dW -> dQ staging
};
// tensor-memory columns (512 allocated); a stage's results are read out before a later stage
// writes their columns (dV and dQ, read out while stages 3 and 5 run, stay clear of them)
constexpr int C_RT = 256, C_DDT = 320;                         // stage 1 (M=128)
constexpr int C_DELTA = 0, C_DTP = 64, C_DW = 128, C_DV = 256;  // stage 2 (delta^T M=128, rest M=64)
constexpr int C_DP = 0, C_Y = 64, C_DQ = 128, C_DK = 384;       // stage 3 (M=64)
constexpr int C_Z = 0, C_KK = 64, C_ZT = 256;                  // stage 4 (M=64)

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
// one step of a recursive-halving sum over lanes l and l ^ o: the lane with bit o set keeps the
// upper M entries, the other the lower M, each adding its partner's copy of them
template <int M>
__device__ __forceinline__ void halve_sum(float (&v)[32], int lane, int o) {
  const bool up = (lane & o) != 0;
#pragma unroll
  for (int i = 0; i < M; ++i) {
    const float send = up ? v[i] : v[i + M];
    const float keep = up ? v[i + M] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
  }
}
// v[0..31] summed over the 16 lanes of each half-warp (all 32 lanes take part): lane l ends with
// the sums of entries 2 (l % 16) and 2 (l % 16) + 1 in v[0] and v[1]
__device__ __forceinline__ void halfwarp_sums(float (&v)[32], int lane) {
  halve_sum<16>(v, lane, 8);
  halve_sum<8>(v, lane, 4);
  halve_sum<4>(v, lane, 2);
  halve_sum<2>(v, lane, 1);
}

__global__ void __launch_bounds__(NG, 1) scan_grad_kernel(
    const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
    const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap gmap,
    const __grid_constant__ CUtensorMap dqmap, const __grid_constant__ CUtensorMap dkmap,
    const __grid_constant__ CUtensorMap dvmap, const bf16* __restrict__ beta, const float* __restrict__ shift,
    int logit, const uint8_t* __restrict__ xt, const uint8_t* __restrict__ hck, const uint8_t* __restrict__ dhck,
    bf16* __restrict__ dbeta, int T, int H, int D, int NC, int total, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t *Vt = sm + GrSmem::VV, *Xt = sm + GrSmem::XX, *Rt = sm + GrSmem::Rt, *dDt = sm + GrSmem::dD;
  uint8_t *Dt = sm + GrSmem::Dt, *Wd = sm + GrSmem::Wd;
  uint8_t *dXt = Rt, *dGt = Rt + TILE_TT, *dVt = dDt, *dPt = Dt, *Yt = Dt + TILE_TT, *dKt = Dt, *dQt = Wd;
  __shared__ float bsm[C], db1[C], db2s[2][C], part[4][C];
  __shared__ uint64_t bar, bar1, la, lb;
  __shared__ uint32_t tbase;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // warps w and w + 4 share tensor-memory lane quadrant w % 4 and split the columns (half)
  const int quarter = warp & 3, half = warp >> 2;
  const int lane128 = quarter * 32 + lane;      // row of an M=128 accumulator
  const int trow = quarter * 16 + (lane & 15);  // token row of an M=64 accumulator (lane < 16)
  const bool rowlane = lane < 16;
  if (tid == 0) {
    // bar: stages 2-5; bar1: stage 1; la: V, P | dH', H, dO | K (three arrivals); lb: T', X | Q
    mbar_init(&bar, 1); mbar_init(&bar1, 1); mbar_init(&la, 3); mbar_init(&lb, 2);
    mbar_fence_init();
  }
  if (warp == 0) { tmem_alloc(&tbase, 512); tmem_relinquish(); }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  const uint32_t lane_tm = taddr(tm, quarter * 32, 0);
  const uint32_t s0 = smem_u32(sm);
  const uint32_t sdH = s0 + GrSmem::DH, sH = s0 + GrSmem::HH, sG = s0 + GrSmem::GG;
  const uint32_t sP = s0 + GrSmem::PP, sT = s0 + GrSmem::TT, sX = s0 + GrSmem::XX, sR = s0 + GrSmem::Rt;
  const uint32_t sdD = s0 + GrSmem::dD, sD = s0 + GrSmem::Dt, sdW = s0 + GrSmem::Wd;
  const uint32_t sdX = sR, sdG = sR + TILE_TT, sdP = sD, sY = sD + TILE_TT;
  // thread 0's account of what it armed or committed and which phases it saw complete: a CTA that
  // stops early waits (bounded) for its copies and products in flight before it returns
  int la_arms = 0, la_seen = 0, lb_arms = 0, lb_seen = 0, b1_commits = 0, b1_seen = 0, b_commits = 0, b_seen = 0;

  struct Coord {
    int b, h, t0;
  };
  auto coords = [&](int chunk) -> Coord {
    const int bh = chunk / NC;
    return Coord{bh / H, bh % H, (chunk - bh * NC) * C};
  };
  auto k_region = [&](int parity) -> uint32_t { return parity ? GrSmem::KB : GrSmem::KA; };
  auto q_region = [&](int parity) -> uint32_t { return parity ? GrSmem::KA : GrSmem::KB; };
  // the loads of chunk `chunk` (thread 0), in the order their regions free up
  auto load_vp = [&](int chunk, const Coord& q) {
    mbar_arrive_expect_tx(&la, TILE_TD + TILE_TT);
    tma_tile(Vt, &vmap, &la, q.h, q.t0, q.b);
    bulk_load(sm + GrSmem::PP, xt + (size_t)chunk * PREP_BYTES + PREP_P, TILE_TT, &la);
    ++la_arms;
  };
  auto load_hg = [&](int chunk, const Coord& q) {
    mbar_arrive_expect_tx(&la, 2 * TILE_JI + TILE_TD);
    bulk_load(sm + GrSmem::DH, dhck + (size_t)chunk * TILE_JI, TILE_JI, &la);
    bulk_load(sm + GrSmem::HH, hck + (size_t)chunk * TILE_JI, TILE_JI, &la);
    tma_tile(sm + GrSmem::GG, &gmap, &la, q.h, q.t0, q.b);
    ++la_arms;
  };
  auto load_k = [&](const Coord& q, int parity) {
    mbar_arrive_expect_tx(&la, TILE_TD);
    tma_tile(sm + k_region(parity), &kmap, &la, q.h, q.t0, q.b);
    ++la_arms;
  };
  auto load_tx = [&](int chunk) {
    const uint8_t* pre = xt + (size_t)chunk * PREP_BYTES;
    mbar_arrive_expect_tx(&lb, 2 * TILE_TT);
    bulk_load(sm + GrSmem::TT, pre + PREP_T, TILE_TT, &lb);
    bulk_load(Xt, pre + PREP_X, TILE_TT, &lb);
    ++lb_arms;
  };
  auto load_q = [&](const Coord& q, int parity) {
    mbar_arrive_expect_tx(&lb, TILE_TD);
    tma_tile(sm + q_region(parity), &qmap, &lb, q.h, q.t0, q.b);
    ++lb_arms;
  };
  // stage 1 of a chunk whose K lives in k_region(parity) (thread 0, after its loads on la)
  auto issue_s1 = [&](int parity) {
    const uint32_t sK = s0 + k_region(parity);
    const uint32_t id = idesc_bf16(128, 64, 0, 0);
    mma_seq<8, 0, 128, 0, 64>(tm + C_RT, sH, sK, id, 0u);    // (K H)^T [j][t]
    mma_seq<8, 0, 128, 0, 64>(tm + C_DDT, sdH, sK, id, 0u);  // ddelta^T = dH'^T K^T + dO^T P
    mma_seq<4, 1, 64, 1, 64>(tm + C_DDT, sG, sP, idesc_bf16(128, 64, 1, 1), 1u);
    umma_commit(&bar1);
    ++b1_commits;
  };
  auto commit = [&]() {
    umma_commit(&bar);
    ++b_commits;
  };
  // all threads: the next phase of bar (thread 0's count sets the parity of everyone's)
  auto wait_mma = [&](bool ok) -> bool {
    if (!ok) return false;
    const bool r = mbar_wait(&bar, (uint32_t)(b_seen & 1));
    if (r) ++b_seen;
    else atomicOr(status, 2);
    tc_fence_after();
    return r;
  };
  auto wait_load = [&](uint64_t* lbar, int& seen) -> bool {
    const bool r = mbar_wait(lbar, (uint32_t)(seen & 1));
    if (r) ++seen;
    else atomicOr(status, 4);
    return r;
  };

  bool ok = true;
  int chunk = blockIdx.x;
  if (tid == 0 && chunk < total) {
    const Coord q = coords(chunk);
    load_vp(chunk, q);
    load_hg(chunk, q);
    load_k(q, 0);
    load_tx(chunk);
    load_q(q, 0);
    if (wait_load(&la, la_seen)) issue_s1(0);
    else ok = false;
  }
  for (int it = 0; chunk < total; chunk += gridDim.x, ++it) {
    const int par = it & 1;
    const int next = chunk + (int)gridDim.x;
    const bool has_next = next < total;
    const Coord cur = coords(chunk), nxt = coords(has_next ? next : chunk);
    const int b = cur.b, h = cur.h, t0 = cur.t0;
    const int valid = min(C, T - t0);
    const int64_t row0 = (int64_t)b * T + t0;
    const uint32_t sK = s0 + k_region(par), sQ = s0 + q_region(par);
    const bf16 bv = fetch_beta(beta + h, row0, H, valid);
    const float bsh = logit ? fetch_shift(shift, row0, valid) : 0.f;
    // stage 1 was issued before this iteration: R^T = V^T - (K H)^T, ddelta^T
    if (ok) {
      const bool r = mbar_wait(&bar1, (uint32_t)(b1_seen & 1));
      if (r) ++b1_seen;
      else { ok = false; atomicOr(status, 2); }
      tc_fence_after();
    }
    {
      float a[32];
      ld32w(lane_tm, C_RT + half * 32, a);
#pragma unroll
      for (int e = 0; e < 32; ++e)
        a[e] = __bfloat162float(*reinterpret_cast<const bf16*>(Vt + sw_offset(64, half * 32 + e, lane128))) - a[e];
      st_row32_bf16(Rt, 128, lane128, half * 32, a);
      ld32w(lane_tm, C_DDT + half * 32, a);
      st_row32_bf16(dDt, 128, lane128, half * 32, a);
    }
    if (tid < C) bsm[tid] = beta_value(bv, logit, bsh);
    if (tid == 0) bulk_wait_read();  // the previous chunk's dQ and dK stores have left Wd and Dt
    publish();
    if (tid == 0 && ok && has_next) load_vp(next, nxt);  // V (also read by the readout above) and P are done
    // stage 2: delta^T = R^T T'^T; dW = -ddelta H^T; dV = T'^T ddelta; dT' = ddelta R^T
    if (tid == 0 && ok) {
      if (wait_load(&lb, lb_seen)) {
        mma_seq<4, 0, 128, 0, 64>(tm + C_DELTA, sR, sT, idesc_bf16(128, 64, 0, 0), 0u);
        mma_seq<8, 1, 128, 1, 128>(tm + C_DW, sdD, sH, idesc_bf16(64, 128, 1, 1, 1), 0u);
        mma_seq<4, 1, 64, 0, 128>(tm + C_DV, sT, sdD, idesc_bf16(64, 128, 1, 0), 0u);
        mma_seq<8, 1, 128, 1, 128>(tm + C_DTP, sdD, sR, idesc_bf16(64, 64, 1, 1), 0u);
        commit();
      } else {
        ok = false;
      }
    }
    ok = wait_mma(ok);
    if (tid != 0 && ok) {  // X is read below (thread 0 saw lb before stage 2)
      const bool r = mbar_wait(&lb, (uint32_t)(lb_seen & 1));
      if (r) ++lb_seen;
      else { ok = false; atomicOr(status, 4); }
    }
    {
      float a[32];
      ld32w(lane_tm, C_DELTA + half * 32, a);
      st_row32_bf16(Dt, 128, lane128, half * 32, a);  // delta^T [j][t]
      float r[64];
      ld64(lane_tm, C_DW + half * 64, r);
      if (rowlane) st_row64_bf16(Wd, 64, trow, half, r);  // dW [t][i]
      // dT' row t: dX = dT' diag(beta) (bf16 operand); dbeta's first part sum_t dT'[t][s] X[t][s]
      float dx[32];
      ld32w(lane_tm, C_DTP + half * 32, a);
#pragma unroll
      for (int c8 = 0; c8 < 4; ++c8) {
        const uint4 xw = *reinterpret_cast<const uint4*>(Xt + sw_chunk(64, trow, half * 4 + c8));
        const bf16* xe = reinterpret_cast<const bf16*>(&xw);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int e = 8 * c8 + i;
          dx[e] = a[e] * bsm[half * 32 + e];
          a[e] = rowlane ? a[e] * __bfloat162float(xe[i]) : 0.f;
        }
      }
      if (rowlane) st_row32_bf16(dXt, 64, trow, half * 32, dx);
      halfwarp_sums(a, lane);
      if (rowlane) {
        part[quarter][half * 32 + 2 * lane] = a[0];
        part[quarter][half * 32 + 2 * lane + 1] = a[1];
      }
    }
    publish();
    // stage 3: dP = dO delta^T; Y = dX X^T; dQ = dO H^T; dK = delta dH'^T
    if (tid == 0 && ok) {
      mma_seq<8, 0, 64, 1, 128>(tm + C_DP, sG, sD, idesc_bf16(64, 64, 0, 1), 0u);
      mma_seq<4, 0, 64, 0, 64>(tm + C_Y, sdX, sX, idesc_bf16(64, 64, 0, 0), 0u);
      mma_seq<8, 0, 64, 1, 128>(tm + C_DQ, sG, sH, idesc_bf16(64, 128, 0, 1), 0u);
      mma_seq<8, 1, 128, 1, 128>(tm + C_DK, sD, sdH, idesc_bf16(64, 128, 1, 1), 0u);
      commit();
    }
    if (tid < C) db1[tid] = (part[0][tid] + part[1][tid]) + (part[2][tid] + part[3][tid]);
    {  // dV, while stage 3 runs: staged over ddelta^T (its products are done)
      float r[64];
      ld64(lane_tm, C_DV + half * 64, r);
      if (rowlane) st_row64_bf16(dVt, 64, trow, half, r);
    }
    ok = wait_mma(ok);
    if (tid == 0 && ok && has_next) load_hg(next, nxt);  // dH', H and dO are done
    {
      float a[32];
      ld32w(lane_tm, C_DP + half * 32, a);
      if (rowlane) {
#pragma unroll
        for (int e = 0; e < 32; ++e) a[e] = half * 32 + e <= trow ? a[e] : 0.f;
        st_row32_bf16(dPt, 64, trow, half * 32, a);
      }
      ld32w(lane_tm, C_Y + half * 32, a);
      if (rowlane) st_row32_bf16(Yt, 64, trow, half * 32, a);
    }
    publish();
    if (tid == 0) store_tile(&dvmap, dVt, h, t0, b, D);
    // stage 4: Z = X^T Y and its transpose; K K^T; dQ += dP K; dK += dP^T Q + T'^T dW
    if (tid == 0 && ok) {
      mma_seq<4, 1, 64, 1, 64>(tm + C_Z, sX, sY, idesc_bf16(64, 64, 1, 1), 0u);
      mma_seq<4, 1, 64, 1, 64>(tm + C_ZT, sY, sX, idesc_bf16(64, 64, 1, 1), 0u);
      mma_seq<8, 0, 64, 0, 64>(tm + C_KK, sK, sK, idesc_bf16(64, 64, 0, 0), 0u);
      mma_seq<4, 0, 64, 1, 64>(tm + C_DQ, sdP, sK, idesc_bf16(64, 128, 0, 1), 1u);
      const uint32_t id_mn = idesc_bf16(64, 128, 1, 1);
      mma_seq<4, 1, 64, 1, 64>(tm + C_DK, sdP, sQ, id_mn, 1u);
      mma_seq<4, 1, 64, 1, 64>(tm + C_DK, sT, sdW, id_mn, 1u);
      commit();
    }
    ok = wait_mma(ok);
    if (tid == 0 && ok && has_next) {  // Q, T' and X are done: the next K lands in Q's region
      load_k(nxt, par ^ 1);
      load_tx(next);
    }
    {
      float z[32], zt[32], kk[32];
      tmem_ld32(lane_tm + (uint32_t)(C_Z + half * 32), z);
      tmem_ld32(lane_tm + (uint32_t)(C_ZT + half * 32), zt);
      tmem_ld32(lane_tm + (uint32_t)(C_KK + half * 32), kk);
      tmem_wait_ld();
      if (rowlane) {
        // dG = diag(beta) dA + (diag(beta) dA)^T has one nonzero term per entry: beta_t dA[t][s]
        // below the diagonal, beta_s dA[s][t] = -beta_s Z^T[t][s] above it
        const float bt = bsm[trow];
        float db2 = 0.f;
#pragma unroll
        for (int e = 0; e < 32; ++e) {  // unconditional loads: a load under the lane test branches
          const int s2 = half * 32 + e;
          const float bs = bsm[s2];
          // 0/1 masks and products rather than selects between computed values
          const float lo = s2 < trow ? 1.f : 0.f, hi = s2 > trow ? 1.f : 0.f;
          const float da = -lo * z[e];
          db2 = fmaf(da, kk[e], db2);
          z[e] = fmaf(bt, da, -hi * bs * zt[e]);
        }
        st_row32_bf16(dGt, 64, trow, half * 32, z);
        db2s[half][trow] = db2;
      }
    }
    publish();
    if (rowlane && half == 0 && trow < valid) {
      const bf16 db = __float2bfloat16_rn(db1[trow] + db2s[0][trow] + db2s[1][trow]);
      // with logits, the gradient through the sigmoid as torch's bf16 sigmoid_backward forms it
      // from the bf16 dbeta and beta: dbeta * (1 - beta) * beta with every intermediate rounded
      // to bf16 (its bf16 arithmetic), so the fused result equals sigmoid-then-scan bit for bit
      const float bt = bsm[trow];
      const float one_minus = __bfloat162float(__float2bfloat16_rn(1.0f - bt));
      const float t = __bfloat162float(__float2bfloat16_rn(__bfloat162float(db) * one_minus));
      dbeta[(row0 + trow) * H + h] = logit ? __float2bfloat16_rn(t * bt) : db;
    }
    // stage 5: dK += dG K; then the next chunk's stage 1 (its columns and regions are free)
    if (tid == 0 && ok) {
      mma_seq<4, 0, 64, 1, 64>(tm + C_DK, sdG, sK, idesc_bf16(64, 128, 0, 1), 1u);
      commit();
      if (has_next) {
        if (wait_load(&la, la_seen)) issue_s1(par ^ 1);
        else ok = false;
      }
    }
    {  // dQ, while stage 5 runs: staged over dW (its products are done)
      float r[64];
      ld64(lane_tm, C_DQ + half * 64, r);
      if (rowlane) st_row64_bf16(dQt, 64, trow, half, r);
    }
    ok = wait_mma(ok);
    if (tid == 0) {
      if (ok && has_next) load_q(nxt, par ^ 1);  // K is done: the next Q lands in its region
      bulk_wait_read();                           // dV has left ddelta^T's region (next stage 1)
    }
    {
      float r[64];
      ld64(lane_tm, C_DK + half * 64, r);
      if (rowlane) st_row64_bf16(dKt, 64, trow, half, r);  // dK staged over dP and Y
    }
    ok = publish_ok(ok);
    if (tid == 0) {
      store_tile(&dqmap, dQt, h, t0, b, D);
      store_tile(&dkmap, dKt, h, t0, b, D);
    }
    if (!ok) break;
  }
  if (tid == 0) {
    // after an early stop: let every armed copy and committed product finish (bounded waits)
    while (la_arms % 3) { mbar_arrive(&la); ++la_arms; }
    while (lb_arms % 2) { mbar_arrive(&lb); ++lb_arms; }
    for (; la_seen < la_arms / 3; ++la_seen) mbar_wait(&la, (uint32_t)(la_seen & 1));
    for (; lb_seen < lb_arms / 2; ++lb_seen) mbar_wait(&lb, (uint32_t)(lb_seen & 1));
    for (; b1_seen < b1_commits; ++b1_seen) mbar_wait(&bar1, (uint32_t)(b1_seen & 1));
    for (; b_seen < b_commits; ++b_seen) mbar_wait(&bar, (uint32_t)(b_seen & 1));
    bulk_wait_read();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
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

namespace {
int scan_bf16_fwd(const void* q, const void* k, const void* v, const void* beta, const float* shift, int logit,
                  const float* state0, void* o, float* state_n, void* saved, int* status, int B, int T, int H,
                  int D, void* stream) {
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
    scan_prep_kernel<<<B * H * NC, NP, sp, st>>>(qm, km, vm, (const bf16*)beta, shift, logit, xt, T, H, NC, status);
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

int scan_bf16_bwd(const void* q, const void* k, const void* v, const void* beta, const float* shift, int logit,
                  const void* saved, const void* dout, const float* dstate_n, void* dq, void* dk, void* dv,
                  void* dbeta, float* dstate0, void* workspace, int* status, int B, int T, int H, int D,
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
    int dev = 0, nsm = 0;
    VB_CUDA_CHECK(cudaGetDevice(&dev), "grad device");
    VB_CUDA_CHECK(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev), "grad SM count");
    const int total = B * H * NC;  // one persistent CTA per SM walks the chunks
    scan_grad_kernel<<<total < nsm ? total : nsm, NG, sg, st>>>(qm, km, vm, gm, dqm, dkm, dvm, (const bf16*)beta,
                                                                 shift, logit, xt, hck, dhck, (bf16*)dbeta, T, H,
                                                                 D, NC, total, status);
    VB_LAUNCH_CHECK("delta_scan_bf16 grad");
  }
  return VB_OK;
}
}  // namespace

extern "C" int vb_delta_scan_bf16_fwd(const void* q, const void* k, const void* v, const void* beta,
                                      const float* state0, void* o, float* state_n, void* saved,
                                      int* status, int B, int T, int H, int D, void* stream) {
  return scan_bf16_fwd(q, k, v, beta, nullptr, 0, state0, o, state_n, saved, status, B, T, H, D, stream);
}

extern "C" int vb_delta_scan_bf16_bwd(const void* q, const void* k, const void* v, const void* beta,
                                      const void* saved, const void* dout, const float* dstate_n,
                                      void* dq, void* dk, void* dv, void* dbeta, float* dstate0,
                                      void* workspace, int* status, int B, int T, int H, int D,
                                      void* stream) {
  return scan_bf16_bwd(q, k, v, beta, nullptr, 0, saved, dout, dstate_n, dq, dk, dv, dbeta, dstate0, workspace,
                       status, B, T, H, D, stream);
}

extern "C" int vb_delta_scan_bf16_fwd_logits(const void* q, const void* k, const void* v, const void* beta_logits,
                                             const float* shift, const float* state0, void* o, float* state_n,
                                             void* saved, int* status, int B, int T, int H, int D, void* stream) {
  VB_REQUIRE(B == 0 || H == 0 || beta_logits != nullptr, "delta_scan_bf16_fwd_logits: null logits");
  return scan_bf16_fwd(q, k, v, beta_logits, shift, 1, state0, o, state_n, saved, status, B, T, H, D, stream);
}

extern "C" int vb_delta_scan_bf16_bwd_logits(const void* q, const void* k, const void* v, const void* beta_logits,
                                             const float* shift, const void* saved, const void* dout,
                                             const float* dstate_n, void* dq, void* dk, void* dv, void* dlogits,
                                             float* dstate0, void* workspace, int* status, int B, int T, int H,
                                             int D, void* stream) {
  return scan_bf16_bwd(q, k, v, beta_logits, shift, 1, saved, dout, dstate_n, dq, dk, dv, dlogits, dstate0,
                       workspace, status, B, T, H, D, stream);
}
