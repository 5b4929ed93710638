// The delta-rule scan in float32, token by token (the contract of vesper/kernels/delta_scan.py:156-187,
// delta_scan_fused_fp32; semantics vesper/recurrence.py:118-163).
//
// Per (batch, head) the state H [key i, value j] is spread over a CTA: lane l of every warp holds
// key rows i = l, l+32, ... and warp w holds value columns j = 32*jb + 4w .. 4w+3 of the CTA's
// column block jb. Per token the two reads of the state (H^T k before the write, H^T q after)
// are warp reductions over i. The backward runs the gradient recurrence in reverse
// (G = dL/dH_t: G += q do^T, dr = beta G^T k, G -= k dr^T) and then the state recurrence forward
// again for the terms that need H (dq = H_t do, dk's H_{t-1} dr); the reductions over value columns
// that span CTAs go through fixed-order partial sums (deterministic).
#include "common.cuh"

namespace vb {
namespace {

// The write strength of token row `row` ((b*T + t)*H + h; `tok` = b*T + t): beta itself, or with
// `logit` set the reference's write_strength, sigmoid(logit + shift[tok]) = 1 / (1 + exp(-x)) in
// float32 as torch.sigmoid forms it (vesper/recurrence.py:34-88).
__device__ __forceinline__ float beta_at(const float* __restrict__ beta, const float* __restrict__ shift, int logit,
                                         int64_t row, int64_t tok) {
  const float raw = __ldg(beta + row);
  if (!logit) return raw;
  const float x = raw + (shift != nullptr ? __ldg(shift + tok) : 0.f);
  return 1.0f / (1.0f + expf(-x));
}
// the same for bfloat16 write strengths: beta (or its logits' sigmoid) rounded to bfloat16, as the
// chunked bfloat16 kernels and torch.sigmoid's bfloat16 output round it
__device__ __forceinline__ float beta_at(const __nv_bfloat16* __restrict__ beta, const float* __restrict__ shift,
                                         int logit, int64_t row, int64_t tok) {
  const float raw = __bfloat162float(beta[row]);
  if (!logit) return raw;
  const float x = raw + (shift != nullptr ? __ldg(shift + tok) : 0.f);
  return __bfloat162float(__float2bfloat16_rn(1.0f / (1.0f + expf(-x))));
}
__device__ __forceinline__ float ld_in(const float* __restrict__ p) { return __ldg(p); }
__device__ __forceinline__ float ld_in(const __nv_bfloat16* __restrict__ p) { return __bfloat162float(*p); }
__device__ __forceinline__ void st_out(float* p, float v) { *p = v; }
__device__ __forceinline__ void st_out(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

constexpr int NWARP = 8;          // warps per CTA
constexpr int CPW = 4;            // value columns per warp
constexpr int BV = NWARP * CPW;   // value columns per CTA

// E: the element type of q, k, v, beta and o (float32, or bfloat16 for the decode step); the
// state and the arithmetic are float32. s0 and sn may be the same buffer (an in-place step): each
// thread reads its state entries before the loop and writes them after it.
template <int NI, typename E>
__global__ void __launch_bounds__(NWARP * 32) scan_f32_fwd_kernel(
    const E* __restrict__ q, const E* __restrict__ k, const E* __restrict__ v,
    const E* __restrict__ beta, const float* __restrict__ shift, int logit, const float* s0,
    E* __restrict__ o, float* sn, float* __restrict__ resid, int T, int H, int D) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jb = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int j0 = jb * BV + warp * CPW;
  float S[NI][CPW];
  const float* s0p = s0 + (int64_t)bh * D * D;
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      S[m][c] = (i < D && j < D) ? s0p[(int64_t)i * D + j] : 0.f;
    }
  }
  // the token's inputs are loaded one token ahead (their latency overlaps the current token's
  // reductions, which are the sequential chain)
  float kk[NI], qq[NI], vv[CPW], bt = 0.f;
  auto load_token = [&](int t, float (&k_)[NI], float (&q_)[NI], float (&v_)[CPW], float& b_) {
    const int64_t row = (((int64_t)b * T + t) * H + h);
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      const int i = lane + 32 * m;
      k_[m] = i < D ? ld_in(k + row * D + i) : 0.f;
      q_[m] = i < D ? ld_in(q + row * D + i) : 0.f;
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c) v_[c] = (j0 + c < D) ? ld_in(v + row * D + j0 + c) : 0.f;
    b_ = beta_at(beta, shift, logit, row, (int64_t)b * T + t);
  };
  if (T > 0) load_token(0, kk, qq, vv, bt);
  for (int t = 0; t < T; ++t) {
    const int64_t row = (((int64_t)b * T + t) * H + h);
    float kn[NI], qn[NI], vn[CPW], bn = 0.f;
    if (t + 1 < T) load_token(t + 1, kn, qn, vn, bn);
    float red[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      float a = 0.f;
#pragma unroll
      for (int m = 0; m < NI; ++m) a = fmaf(S[m][c], kk[m], a);
      red[c] = a;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int c = 0; c < CPW; ++c) red[c] += __shfl_xor_sync(0xffffffffu, red[c], off);
    float r[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) r[c] = vv[c] - red[c];
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      const float bk = bt * kk[m];
#pragma unroll
      for (int c = 0; c < CPW; ++c) S[m][c] = fmaf(bk, r[c], S[m][c]);
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      float a = 0.f;
#pragma unroll
      for (int m = 0; m < NI; ++m) a = fmaf(S[m][c], qq[m], a);
      red[c] = a;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int c = 0; c < CPW; ++c) red[c] += __shfl_xor_sync(0xffffffffu, red[c], off);
    if (lane < CPW) {
      float ov = red[0], rv = r[0];
#pragma unroll
      for (int c = 1; c < CPW; ++c)
        if (lane == c) { ov = red[c]; rv = r[c]; }
      const int j = j0 + lane;
      if (j < D) {
        st_out(o + row * D + j, ov);
        if (resid) resid[row * D + j] = rv;
      }
    }
    if (t + 1 < T) {
#pragma unroll
      for (int m = 0; m < NI; ++m) { kk[m] = kn[m]; qq[m] = qn[m]; }
#pragma unroll
      for (int c = 0; c < CPW; ++c) vv[c] = vn[c];
      bt = bn;
    }
  }
  float* snp = sn + (int64_t)bh * D * D;
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      if (i < D && j < D) snp[(int64_t)i * D + j] = S[m][c];
    }
  }
}

// Sums one [D] vector over the CTA's warps (warp order) into out[D]; red: smem [NWARP][D].
template <int NI>
__device__ __forceinline__ void cta_sum_store(float (&part)[NI], float* red, float* out, int D) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
    if (i < D) red[warp * D + i] = part[m];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < D; i += blockDim.x) {
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) a += red[w * D + i];
    out[i] = a;
  }
  __syncthreads();
}

// Phase A (reverse): G, dv, the partial of G r over this CTA's columns, dstate0.
// Phase B (forward): the partials of H_{t-1} dr and H_t do over this CTA's columns.
// part: [3][NJB][B*T*H][D] = (G r, H_{t-1} dr, H_t do).
template <int NI>
__global__ void __launch_bounds__(NWARP * 32) scan_f32_bwd_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ beta,
    const float* __restrict__ shift, int logit,
    const float* __restrict__ s0, const float* __restrict__ resid, const float* __restrict__ dout,
    const float* __restrict__ dsn, float* __restrict__ dv, float* __restrict__ ds0,
    float* __restrict__ part, int B, int T, int H, int D) {
  extern __shared__ float red[];  // [NWARP][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jb = blockIdx.x, NJB = gridDim.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int j0 = jb * BV + warp * CPW;
  const int64_t rows = (int64_t)B * T * H;
  float* part_gr = part + ((int64_t)0 * NJB + jb) * rows * D;
  float* part_hd = part + ((int64_t)1 * NJB + jb) * rows * D;
  float* part_dq = part + ((int64_t)2 * NJB + jb) * rows * D;
  float G[NI][CPW];
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      G[m][c] = (dsn && i < D && j < D) ? dsn[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
    }
  }
  // phase A: a token's inputs are loaded one token ahead (reverse order)
  auto load_a = [&](int t, float (&k_)[NI], float (&q_)[NI], float (&g_)[CPW], float (&r_)[CPW], float& b_) {
    const int64_t row = (((int64_t)b * T + t) * H + h);
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      const int i = lane + 32 * m;
      k_[m] = i < D ? __ldg(k + row * D + i) : 0.f;
      q_[m] = i < D ? __ldg(q + row * D + i) : 0.f;
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const bool ok = j0 + c < D;
      g_[c] = ok ? __ldg(dout + row * D + j0 + c) : 0.f;
      r_[c] = ok ? __ldg(resid + row * D + j0 + c) : 0.f;
    }
    b_ = beta_at(beta, shift, logit, row, (int64_t)b * T + t);
  };
  float kk[NI], qq[NI], gg[CPW], rr[CPW], bt = 0.f;
  if (T > 0) load_a(T - 1, kk, qq, gg, rr, bt);
  for (int t = T - 1; t >= 0; --t) {
    const int64_t row = (((int64_t)b * T + t) * H + h);
    float kn[NI], qn[NI], gn[CPW], rn[CPW], bn = 0.f;
    if (t > 0) load_a(t - 1, kn, qn, gn, rn, bn);
#pragma unroll
    for (int m = 0; m < NI; ++m)
#pragma unroll
      for (int c = 0; c < CPW; ++c) G[m][c] = fmaf(qq[m], gg[c], G[m][c]);
    float red_c[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      float a = 0.f;
#pragma unroll
      for (int m = 0; m < NI; ++m) a = fmaf(G[m][c], kk[m], a);
      red_c[c] = a;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int c = 0; c < CPW; ++c) red_c[c] += __shfl_xor_sync(0xffffffffu, red_c[c], off);
    float dr[CPW];
#pragma unroll
    for (int c = 0; c < CPW; ++c) dr[c] = bt * red_c[c];
    if (lane < CPW) {
      float x = dr[0];
#pragma unroll
      for (int c = 1; c < CPW; ++c)
        if (lane == c) x = dr[c];
      if (j0 + lane < D) dv[row * D + j0 + lane] = x;
    }
    float gr[NI];
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      float a = 0.f;
#pragma unroll
      for (int c = 0; c < CPW; ++c) a = fmaf(G[m][c], rr[c], a);
      gr[m] = a;
    }
    cta_sum_store<NI>(gr, red, part_gr + row * D, D);
#pragma unroll
    for (int m = 0; m < NI; ++m)
#pragma unroll
      for (int c = 0; c < CPW; ++c) G[m][c] = fmaf(-kk[m], dr[c], G[m][c]);
    if (t > 0) {
#pragma unroll
      for (int m = 0; m < NI; ++m) { kk[m] = kn[m]; qq[m] = qn[m]; }
#pragma unroll
      for (int c = 0; c < CPW; ++c) { gg[c] = gn[c]; rr[c] = rn[c]; }
      bt = bn;
    }
  }
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      if (i < D && j < D) ds0[(int64_t)bh * D * D + (int64_t)i * D + j] = G[m][c];
    }
  }
  __syncthreads();  // dv of this CTA's columns is complete before phase B reads it back
  float S[NI][CPW];
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      S[m][c] = (i < D && j < D) ? s0[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
    }
  }
  // phase B: likewise one token ahead (forward order); dv of this CTA's columns was written above
  auto load_b = [&](int t, float (&k_)[NI], float (&g_)[CPW], float (&r_)[CPW], float (&d_)[CPW], float& b_) {
    const int64_t row = (((int64_t)b * T + t) * H + h);
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      const int i = lane + 32 * m;
      k_[m] = i < D ? __ldg(k + row * D + i) : 0.f;
    }
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const bool ok = j0 + c < D;
      g_[c] = ok ? __ldg(dout + row * D + j0 + c) : 0.f;
      r_[c] = ok ? __ldg(resid + row * D + j0 + c) : 0.f;
      d_[c] = ok ? dv[row * D + j0 + c] : 0.f;
    }
    b_ = beta_at(beta, shift, logit, row, (int64_t)b * T + t);
  };
  float dr[CPW];
  if (T > 0) load_b(0, kk, gg, rr, dr, bt);
  for (int t = 0; t < T; ++t) {
    const int64_t row = (((int64_t)b * T + t) * H + h);
    float kn[NI], gn[CPW], rn[CPW], dn[CPW], bn = 0.f;
    if (t + 1 < T) load_b(t + 1, kn, gn, rn, dn, bn);
    float hd[NI];
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      float a = 0.f;
#pragma unroll
      for (int c = 0; c < CPW; ++c) a = fmaf(S[m][c], dr[c], a);
      hd[m] = a;
    }
    cta_sum_store<NI>(hd, red, part_hd + row * D, D);
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      const float bk = bt * kk[m];
#pragma unroll
      for (int c = 0; c < CPW; ++c) S[m][c] = fmaf(bk, rr[c], S[m][c]);
    }
    float dq[NI];
#pragma unroll
    for (int m = 0; m < NI; ++m) {
      float a = 0.f;
#pragma unroll
      for (int c = 0; c < CPW; ++c) a = fmaf(S[m][c], gg[c], a);
      dq[m] = a;
    }
    cta_sum_store<NI>(dq, red, part_dq + row * D, D);
    if (t + 1 < T) {
#pragma unroll
      for (int m = 0; m < NI; ++m) kk[m] = kn[m];
#pragma unroll
      for (int c = 0; c < CPW; ++c) { gg[c] = gn[c]; rr[c] = rn[c]; dr[c] = dn[c]; }
      bt = bn;
    }
  }
}

// Per (b, t, h): sums the column-block partials in order; dk = beta * Gr - H dr, dbeta = k . Gr.
// With logits, dbeta is the gradient of the logits: (dbeta * (1 - beta)) * beta, the order of
// torch's sigmoid_backward.
__global__ void scan_f32_finish_kernel(const float* __restrict__ k, const float* __restrict__ beta,
                                       const float* __restrict__ shift, int logit,
                                       const float* __restrict__ part, float* __restrict__ dq,
                                       float* __restrict__ dk, float* __restrict__ dbeta,
                                       int64_t rows, int H, int D, int NJB) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float bt = beta_at(beta, shift, logit, row, row / H);
  float dotk = 0.f;
  for (int i = lane; i < D; i += 32) {
    float gr = 0.f, hd = 0.f, qd = 0.f;
    for (int jb = 0; jb < NJB; ++jb) {
      gr += part[((int64_t)0 * NJB + jb) * rows * D + row * D + i];
      hd += part[((int64_t)1 * NJB + jb) * rows * D + row * D + i];
      qd += part[((int64_t)2 * NJB + jb) * rows * D + row * D + i];
    }
    dq[row * D + i] = qd;
    dk[row * D + i] = bt * gr - hd;
    dotk = fmaf(k[row * D + i], gr, dotk);
  }
  dotk = warp_sum(dotk);
  if (lane == 0) dbeta[row] = logit ? (dotk * (1.0f - bt)) * bt : dotk;
}

// ---- staged variants (head width a multiple of 4) ---------------------------------------------
// The same recurrences, arithmetic and orders as the kernels above, with the inputs of TB-token
// blocks copied into a CTA-shared ring by cp.async NBUF blocks ahead of their use (one barrier
// pair per block instead of a load on every token's dependent chain), and the backward's
// reductions over the CTA's warps buffered per block (the per-token CTA barriers of
// cta_sum_store become two per block): every partial sum is formed in the same order.
constexpr int TB = 8;    // tokens per staged block
constexpr int NBUF = 4;  // blocks in flight

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// the write strength of a staged token: the raw value, or with `logit` the sigmoid of it plus the
// shift, as beta_at forms it
__device__ __forceinline__ float staged_beta(const float* rec_b, int logit, bool has_shift) {
  const float raw = rec_b[0];
  if (!logit) return raw;
  const float x = raw + (has_shift ? rec_b[1] : 0.f);
  return 1.0f / (1.0f + expf(-x));
}

// Copies the rows of tokens [t0, t0 + TB) named by `vecs` (each a float row pointer, an offset into
// the record and a count of 16-byte chunks) plus beta and the shift into one ring slot.
struct StageRow {
  const float* src;  // row of token t0 (advanced by `stride` floats per token)
  int64_t stride;
  int at;            // float offset in a token's record
  int chunks;        // 16-byte chunks per token
};

template <int NROWS>
__device__ __forceinline__ void stage_block(float* slot, int REC, int t0, int T, const StageRow (&rows)[NROWS],
                                            const float* beta_p, const float* shift_p, int64_t beta_stride,
                                            int BOFF) {
  int per = 0;
#pragma unroll
  for (int r = 0; r < NROWS; ++r) per += rows[r].chunks;
  for (int c = threadIdx.x; c < TB * per; c += NWARP * 32) {
    const int tt = c / per, t = t0 + tt;
    if (t >= T) continue;
    int w = c - tt * per;
#pragma unroll
    for (int r = 0; r < NROWS; ++r) {
      if (w >= 0 && w < rows[r].chunks) cp_async16(slot + tt * REC + rows[r].at + 4 * w, rows[r].src + (int64_t)t * rows[r].stride + 4 * w);
      w -= rows[r].chunks;
    }
  }
  for (int tt = threadIdx.x; tt < TB; tt += NWARP * 32) {
    const int t = t0 + tt;
    if (t >= T) continue;
    cp_async4(slot + tt * REC + BOFF, beta_p + (int64_t)t * beta_stride);
    if (shift_p != nullptr) cp_async4(slot + tt * REC + BOFF + 1, shift_p + t);
  }
}

template <int NI>
__global__ void __launch_bounds__(NWARP * 32) scan_f32_fwd_staged_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ beta, const float* __restrict__ shift, int logit, const float* s0,
    float* __restrict__ o, float* sn, float* __restrict__ resid, int T, int H, int D) {
  extern __shared__ __align__(16) float ring[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jb = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int j0 = jb * BV + warp * CPW;
  const int ncol = min(BV, D - jb * BV);
  const int REC = 2 * D + BV + 4;  // k, q, this CTA's v columns, beta and shift
  float S[NI][CPW];
  const float* s0p = s0 + (int64_t)bh * D * D;
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      S[m][c] = (i < D && j < D) ? s0p[(int64_t)i * D + j] : 0.f;
    }
  }
  const int64_t row0 = (int64_t)b * T * H + h;  // token t's row is row0 + t * H
  const int64_t rs = (int64_t)H * D;
  const StageRow rows[3] = {{k + row0 * D, rs, 0, D / 4}, {q + row0 * D, rs, D, D / 4},
                            {v + row0 * D + jb * BV, rs, 2 * D, ncol / 4}};
  const float* shift_p = (logit && shift != nullptr) ? shift + (int64_t)b * T : nullptr;
  const int NBLK = (T + TB - 1) / TB;
  auto slot = [&](int blk) { return ring + (blk % NBUF) * TB * REC; };
#pragma unroll 1
  for (int i = 0; i < NBUF; ++i) {
    if (i < NBLK) stage_block<3>(slot(i), REC, i * TB, T, rows, beta + row0, shift_p, H, 2 * D + BV);
    cp_commit();
  }
  for (int blk = 0; blk < NBLK; ++blk) {
    cp_wait<NBUF - 1>();
    __syncthreads();  // every thread's copies of this block are visible
    const float* sl = slot(blk);
    const int tn = min(TB, T - blk * TB);
    for (int tt = 0; tt < tn; ++tt) {
      const int t = blk * TB + tt;
      const float* rec = sl + tt * REC;
      float kk[NI], qq[NI], vv[CPW];
#pragma unroll
      for (int m = 0; m < NI; ++m) {
        const int i = lane + 32 * m;
        kk[m] = i < D ? rec[i] : 0.f;
        qq[m] = i < D ? rec[D + i] : 0.f;
      }
#pragma unroll
      for (int c = 0; c < CPW; ++c) vv[c] = (j0 + c < D) ? rec[2 * D + warp * CPW + c] : 0.f;
      const float bt = staged_beta(rec + 2 * D + BV, logit, shift_p != nullptr);
      const int64_t row = row0 + (int64_t)t * H;
      float red[CPW];
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        float a = 0.f;
#pragma unroll
        for (int m = 0; m < NI; ++m) a = fmaf(S[m][c], kk[m], a);
        red[c] = a;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int c = 0; c < CPW; ++c) red[c] += __shfl_xor_sync(0xffffffffu, red[c], off);
      float r[CPW];
#pragma unroll
      for (int c = 0; c < CPW; ++c) r[c] = vv[c] - red[c];
#pragma unroll
      for (int m = 0; m < NI; ++m) {
        const float bk = bt * kk[m];
#pragma unroll
        for (int c = 0; c < CPW; ++c) S[m][c] = fmaf(bk, r[c], S[m][c]);
      }
#pragma unroll
      for (int c = 0; c < CPW; ++c) {
        float a = 0.f;
#pragma unroll
        for (int m = 0; m < NI; ++m) a = fmaf(S[m][c], qq[m], a);
        red[c] = a;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1)
#pragma unroll
        for (int c = 0; c < CPW; ++c) red[c] += __shfl_xor_sync(0xffffffffu, red[c], off);
      if (lane < CPW) {
        float ov = red[0], rv = r[0];
#pragma unroll
        for (int c = 1; c < CPW; ++c)
          if (lane == c) { ov = red[c]; rv = r[c]; }
        const int j = j0 + lane;
        if (j < D) {
          o[row * D + j] = ov;
          if (resid) resid[row * D + j] = rv;
        }
      }
    }
    __syncthreads();  // every warp has read the slot: it takes block blk + NBUF
    if (blk + NBUF < NBLK) stage_block<3>(slot(blk), REC, (blk + NBUF) * TB, T, rows, beta + row0, shift_p, H, 2 * D + BV);
    cp_commit();
  }
  cp_wait<0>();
  float* snp = sn + (int64_t)bh * D * D;
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      if (i < D && j < D) snp[(int64_t)i * D + j] = S[m][c];
    }
  }
}

// Forward, lanes split over (row group, column): lane l = 4 g + c holds rows [g R, g R + R) (R = D/8)
// of column j0 + c of the state, so each token's two reductions over the key index are R local
// products and three shuffle levels (xor 4, 8, 16) instead of five levels over four columns: the
// shuffle unit, not the chain, had bounded the row layout above. Every sum is a different order of
// the same float32 products (within float32 rounding of the row layout's).
template <int R>
__global__ void __launch_bounds__(NWARP * 32) scan_f32_fwd_group_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    const float* __restrict__ beta, const float* __restrict__ shift, int logit, const float* s0,
    float* __restrict__ o, float* sn, float* __restrict__ resid, int T, int H, int D) {
  extern __shared__ __align__(16) float ring[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int jb = blockIdx.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int j = jb * BV + warp * CPW + c;  // this lane's column
  const bool jlive = j < D;
  const int ncol = min(BV, D - jb * BV);
  const int REC = 2 * D + BV + 4;  // k, q, this CTA's v columns, beta and shift
  float S[R];
  const float* s0p = s0 + (int64_t)bh * D * D;
#pragma unroll
  for (int r = 0; r < R; ++r) S[r] = jlive ? s0p[(int64_t)(g * R + r) * D + j] : 0.f;
  const int64_t row0 = (int64_t)b * T * H + h;
  const int64_t rs = (int64_t)H * D;
  const StageRow rows[3] = {{k + row0 * D, rs, 0, D / 4}, {q + row0 * D, rs, D, D / 4},
                            {v + row0 * D + jb * BV, rs, 2 * D, ncol / 4}};
  const float* shift_p = (logit && shift != nullptr) ? shift + (int64_t)b * T : nullptr;
  const int NBLK = (T + TB - 1) / TB;
  auto slot = [&](int blk) { return ring + (blk % NBUF) * TB * REC; };
#pragma unroll 1
  for (int i = 0; i < NBUF; ++i) {
    if (i < NBLK) stage_block<3>(slot(i), REC, i * TB, T, rows, beta + row0, shift_p, H, 2 * D + BV);
    cp_commit();
  }
  float pq[R];  // the previous token's query: its output is reduced with this token's read
#pragma unroll
  for (int r = 0; r < R; ++r) pq[r] = 0.f;
  int64_t prow = -1;  // the previous token's row (none yet)
  float prv = 0.f;
  for (int blk = 0; blk < NBLK; ++blk) {
    cp_wait<NBUF - 1>();
    __syncthreads();
    const float* sl = slot(blk);
    const int tn = min(TB, T - blk * TB);
    for (int tt = 0; tt < tn; ++tt) {
      const int t = blk * TB + tt;
      const float* rec = sl + tt * REC;
      float kk[R], qq[R];
#pragma unroll
      for (int r = 0; r < R; r += (R % 4 == 0 ? 4 : 1)) {
        if constexpr (R % 4 == 0) {
          const float4 a = *reinterpret_cast<const float4*>(rec + g * R + r);
          const float4 e = *reinterpret_cast<const float4*>(rec + D + g * R + r);
          kk[r] = a.x; kk[r + 1] = a.y; kk[r + 2] = a.z; kk[r + 3] = a.w;
          qq[r] = e.x; qq[r + 1] = e.y; qq[r + 2] = e.z; qq[r + 3] = e.w;
        } else {
          kk[r] = rec[g * R + r];
          qq[r] = rec[D + g * R + r];
        }
      }
      const float vv = jlive ? rec[2 * D + warp * CPW + c] : 0.f;
      const float bt = staged_beta(rec + 2 * D + BV, logit, shift_p != nullptr);
      // token t's read H^T k and token t-1's output H^T q use the same state (after t-1's write):
      // one pass of three shuffle levels reduces both (two partial sums each: half the chain)
      float a0 = 0.f, a1 = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        if (r & 1) { a1 = fmaf(S[r], kk[r], a1); o1 = fmaf(S[r], pq[r], o1); }
        else { a0 = fmaf(S[r], kk[r], a0); o0 = fmaf(S[r], pq[r], o0); }
      }
      float red = a0 + a1, ov = o0 + o1;
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        red += __shfl_xor_sync(0xffffffffu, red, off);
        ov += __shfl_xor_sync(0xffffffffu, ov, off);
      }
      if (prow >= 0 && g == 0 && jlive) {
        o[prow * D + j] = ov;
        if (resid) resid[prow * D + j] = prv;
      }
      const float rv = vv - red;
      const float br = bt * rv;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        S[r] = fmaf(kk[r], br, S[r]);
        pq[r] = qq[r];
      }
      prow = row0 + (int64_t)t * H;
      prv = rv;
    }
    __syncthreads();
    if (blk + NBUF < NBLK) stage_block<3>(slot(blk), REC, (blk + NBUF) * TB, T, rows, beta + row0, shift_p, H, 2 * D + BV);
    cp_commit();
  }
  cp_wait<0>();
  if (prow >= 0) {  // the last token's output
    float o0 = 0.f, o1 = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (r & 1) o1 = fmaf(S[r], pq[r], o1);
      else o0 = fmaf(S[r], pq[r], o0);
    }
    float ov = o0 + o1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) ov += __shfl_xor_sync(0xffffffffu, ov, off);
    if (g == 0 && jlive) {
      o[prow * D + j] = ov;
      if (resid) resid[prow * D + j] = prv;
    }
  }
  if (jlive) {
    float* snp = sn + (int64_t)bh * D * D;
#pragma unroll
    for (int r = 0; r < R; ++r) snp[(int64_t)(g * R + r) * D + j] = S[r];
  }
}

// Adds one token's per-warp partials (NI per lane over i) of the CTA's buffered block into
// part[row][i] in warp order, for the block's tn tokens; buf: [TB][NWARP][D].
__device__ __forceinline__ void flush_partials(const float* buf, float* part, int64_t row0, int64_t H, int t0,
                                               int tn, int D) {
  for (int e = threadIdx.x; e < tn * D; e += NWARP * 32) {
    const int tt = e / D, i = e - tt * D;
    float a = 0.f;
#pragma unroll
    for (int w = 0; w < NWARP; ++w) a += buf[(tt * NWARP + w) * D + i];
    part[(row0 + (int64_t)(t0 + tt) * H) * D + i] = a;
  }
}

// GA: phase A in the (row group, column) lane layout of scan_f32_fwd_group_kernel (D = 32 NI):
// the reduction over the key index takes three shuffle levels, the one over the CTA's columns two
// recursive-halving levels and the warp buffer; phase B keeps the row layout, whose reductions
// over columns are local.
template <int NI, bool GA>
__global__ void __launch_bounds__(NWARP * 32) scan_f32_bwd_staged_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ beta,
    const float* __restrict__ shift, int logit,
    const float* __restrict__ s0, const float* __restrict__ resid, const float* __restrict__ dout,
    const float* __restrict__ dsn, float* __restrict__ dv, float* __restrict__ ds0,
    float* __restrict__ part, int B, int T, int H, int D) {
  extern __shared__ __align__(16) float smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int jb = blockIdx.x, NJB = gridDim.x, bh = blockIdx.y, b = bh / H, h = bh % H;
  const int j0 = jb * BV + warp * CPW;
  const int ncol = min(BV, D - jb * BV);
  const int64_t rows = (int64_t)B * T * H;
  float* part_gr = part + ((int64_t)0 * NJB + jb) * rows * D;
  float* part_hd = part + ((int64_t)1 * NJB + jb) * rows * D;
  float* part_dq = part + ((int64_t)2 * NJB + jb) * rows * D;
  const int REC = 2 * D + 3 * BV + 4;  // k, q, g, r, dv (this CTA's columns), beta and shift
  float* ring = smem;
  float* buf = smem + NBUF * TB * REC;  // [2][TB][NWARP][D] partials of a block
  float* buf1 = buf + TB * NWARP * D;
  const int64_t row0 = (int64_t)b * T * H + h;
  const int64_t rs = (int64_t)H * D;
  const float* shift_p = (logit && shift != nullptr) ? shift + (int64_t)b * T : nullptr;
  const int NBLK = (T + TB - 1) / TB;
  auto slot = [&](int i) { return ring + (i % NBUF) * TB * REC; };
  if constexpr (GA) {
    // ---- phase A, (row group, column) layout: lane = 4 g + c holds rows [g R, g R + R) of column jc
    constexpr int R = 4 * NI;
    const int g = lane >> 2, c = lane & 3;
    const int jc = jb * BV + warp * CPW + c;
    const bool jlive = jc < D;
    float G[R];
#pragma unroll
    for (int r = 0; r < R; ++r) G[r] = (dsn && jlive) ? dsn[(int64_t)bh * D * D + (int64_t)(g * R + r) * D + jc] : 0.f;
    const StageRow rows_a[4] = {{k + row0 * D, rs, 0, D / 4}, {q + row0 * D, rs, D, D / 4},
                                {dout + row0 * D + jb * BV, rs, 2 * D, ncol / 4},
                                {resid + row0 * D + jb * BV, rs, 2 * D + BV, ncol / 4}};
#pragma unroll 1
    for (int i = 0; i < NBUF; ++i) {
      if (i < NBLK) stage_block<4>(slot(i), REC, (NBLK - 1 - i) * TB, T, rows_a, beta + row0, shift_p, H, 2 * D + 3 * BV);
      cp_commit();
    }
    // this lane's rows of the CTA-column sums after two halving levels (xor 1, then xor 2)
    const int rbase = g * R + (c & 1) * (R / 2) + ((c >> 1) & 1) * (R / 4);
    for (int i = 0; i < NBLK; ++i) {
      const int blk = NBLK - 1 - i, t0 = blk * TB, tn = min(TB, T - t0);
      cp_wait<NBUF - 1>();
      __syncthreads();
      const float* sl = slot(i);
      for (int tt = tn - 1; tt >= 0; --tt) {
        const int t = t0 + tt;
        const float* rec = sl + tt * REC;
        float kk[R], qq[R];
#pragma unroll
        for (int r = 0; r < R; r += 4) {
          const float4 a = *reinterpret_cast<const float4*>(rec + g * R + r);
          const float4 e = *reinterpret_cast<const float4*>(rec + D + g * R + r);
          kk[r] = a.x; kk[r + 1] = a.y; kk[r + 2] = a.z; kk[r + 3] = a.w;
          qq[r] = e.x; qq[r + 1] = e.y; qq[r + 2] = e.z; qq[r + 3] = e.w;
        }
        const float gg = jlive ? rec[2 * D + warp * CPW + c] : 0.f;
        const float rr = jlive ? rec[2 * D + BV + warp * CPW + c] : 0.f;
        const float bt = staged_beta(rec + 2 * D + 3 * BV, logit, shift_p != nullptr);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          G[r] = fmaf(qq[r], gg, G[r]);
          if (r & 1) a1 = fmaf(G[r], kk[r], a1);
          else a0 = fmaf(G[r], kk[r], a0);
        }
        // the read H^T k (three levels over the row groups) and gr = G r over the warp's four
        // columns (recursive halving, xor 1 then xor 2) are independent: their shuffles interleave
        float red = a0 + a1;
        float p[R];
#pragma unroll
        for (int r = 0; r < R; ++r) p[r] = G[r] * rr;
        red += __shfl_xor_sync(0xffffffffu, red, 4);
        {
          const bool up = (lane & 1) != 0;
#pragma unroll
          for (int r = 0; r < R / 2; ++r) {
            const float send = up ? p[r] : p[r + R / 2];
            const float keep = up ? p[r + R / 2] : p[r];
            p[r] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
          }
        }
        red += __shfl_xor_sync(0xffffffffu, red, 8);
        {
          const bool up = (lane & 2) != 0;
#pragma unroll
          for (int r = 0; r < R / 4; ++r) {
            const float send = up ? p[r] : p[r + R / 4];
            const float keep = up ? p[r + R / 4] : p[r];
            p[r] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
          }
        }
        red += __shfl_xor_sync(0xffffffffu, red, 16);
        const float dr = bt * red;
        if (g == 0 && jlive) dv[(row0 + (int64_t)t * H) * D + jc] = dr;
#pragma unroll
        for (int r = 0; r < R / 4; ++r) buf[(tt * NWARP + warp) * D + rbase + r] = p[r];
#pragma unroll
        for (int r = 0; r < R; ++r) G[r] = fmaf(-kk[r], dr, G[r]);
      }
      __syncthreads();  // the slot is read and the block's partials are in buf
      flush_partials(buf, part_gr, row0, H, t0, tn, D);
      if (i + NBUF < NBLK) stage_block<4>(slot(i), REC, (NBLK - 1 - (i + NBUF)) * TB, T, rows_a, beta + row0, shift_p, H, 2 * D + 3 * BV);
      cp_commit();
      __syncthreads();  // buf is free again
    }
    cp_wait<0>();
    if (jlive) {
#pragma unroll
      for (int r = 0; r < R; ++r) ds0[(int64_t)bh * D * D + (int64_t)(g * R + r) * D + jc] = G[r];
    }
  } else {
    float G[NI][CPW];
  #pragma unroll
    for (int m = 0; m < NI; ++m) {
      const int i = lane + 32 * m;
  #pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int j = j0 + c;
        G[m][c] = (dsn && i < D && j < D) ? dsn[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
      }
    }
    // phase A, blocks in reverse: block i of the walk is block NBLK - 1 - i of the sequence
    {
      const StageRow rows_a[4] = {{k + row0 * D, rs, 0, D / 4}, {q + row0 * D, rs, D, D / 4},
                                  {dout + row0 * D + jb * BV, rs, 2 * D, ncol / 4},
                                  {resid + row0 * D + jb * BV, rs, 2 * D + BV, ncol / 4}};
  #pragma unroll 1
      for (int i = 0; i < NBUF; ++i) {
        if (i < NBLK) stage_block<4>(slot(i), REC, (NBLK - 1 - i) * TB, T, rows_a, beta + row0, shift_p, H, 2 * D + 3 * BV);
        cp_commit();
      }
      for (int i = 0; i < NBLK; ++i) {
        const int blk = NBLK - 1 - i, t0 = blk * TB, tn = min(TB, T - t0);
        cp_wait<NBUF - 1>();
        __syncthreads();
        const float* sl = slot(i);
        for (int tt = tn - 1; tt >= 0; --tt) {
          const int t = t0 + tt;
          const float* rec = sl + tt * REC;
          float kk[NI], qq[NI], gg[CPW], rr[CPW];
  #pragma unroll
          for (int m = 0; m < NI; ++m) {
            const int ii = lane + 32 * m;
            kk[m] = ii < D ? rec[ii] : 0.f;
            qq[m] = ii < D ? rec[D + ii] : 0.f;
          }
  #pragma unroll
          for (int c = 0; c < CPW; ++c) {
            const bool ok = j0 + c < D;
            gg[c] = ok ? rec[2 * D + warp * CPW + c] : 0.f;
            rr[c] = ok ? rec[2 * D + BV + warp * CPW + c] : 0.f;
          }
          const float bt = staged_beta(rec + 2 * D + 3 * BV, logit, shift_p != nullptr);
          const int64_t row = row0 + (int64_t)t * H;
  #pragma unroll
          for (int m = 0; m < NI; ++m)
  #pragma unroll
            for (int c = 0; c < CPW; ++c) G[m][c] = fmaf(qq[m], gg[c], G[m][c]);
          float red_c[CPW];
  #pragma unroll
          for (int c = 0; c < CPW; ++c) {
            float a = 0.f;
  #pragma unroll
            for (int m = 0; m < NI; ++m) a = fmaf(G[m][c], kk[m], a);
            red_c[c] = a;
          }
  #pragma unroll
          for (int off = 16; off > 0; off >>= 1)
  #pragma unroll
            for (int c = 0; c < CPW; ++c) red_c[c] += __shfl_xor_sync(0xffffffffu, red_c[c], off);
          float dr[CPW];
  #pragma unroll
          for (int c = 0; c < CPW; ++c) dr[c] = bt * red_c[c];
          if (lane < CPW) {
            float x = dr[0];
  #pragma unroll
            for (int c = 1; c < CPW; ++c)
              if (lane == c) x = dr[c];
            if (j0 + lane < D) dv[row * D + j0 + lane] = x;
          }
  #pragma unroll
          for (int m = 0; m < NI; ++m) {
            float a = 0.f;
  #pragma unroll
            for (int c = 0; c < CPW; ++c) a = fmaf(G[m][c], rr[c], a);
            const int ii = lane + 32 * m;
            if (ii < D) buf[(tt * NWARP + warp) * D + ii] = a;
          }
  #pragma unroll
          for (int m = 0; m < NI; ++m)
  #pragma unroll
            for (int c = 0; c < CPW; ++c) G[m][c] = fmaf(-kk[m], dr[c], G[m][c]);
        }
        __syncthreads();  // the slot is read and the block's partials are in buf
        flush_partials(buf, part_gr, row0, H, t0, tn, D);
        if (i + NBUF < NBLK) stage_block<4>(slot(i), REC, (NBLK - 1 - (i + NBUF)) * TB, T, rows_a, beta + row0, shift_p, H, 2 * D + 3 * BV);
        cp_commit();
        __syncthreads();  // buf is free again
      }
      cp_wait<0>();
    }
  #pragma unroll
    for (int m = 0; m < NI; ++m) {
      const int i = lane + 32 * m;
  #pragma unroll
      for (int c = 0; c < CPW; ++c) {
        const int j = j0 + c;
        if (i < D && j < D) ds0[(int64_t)bh * D * D + (int64_t)i * D + j] = G[m][c];
      }
    }
  }
  __syncthreads();  // dv of this CTA's columns is complete before phase B copies it back
  float S[NI][CPW];
#pragma unroll
  for (int m = 0; m < NI; ++m) {
    const int i = lane + 32 * m;
#pragma unroll
    for (int c = 0; c < CPW; ++c) {
      const int j = j0 + c;
      S[m][c] = (i < D && j < D) ? s0[(int64_t)bh * D * D + (int64_t)i * D + j] : 0.f;
    }
  }
  // phase B, blocks forward: k, g, r, dv
  {
    const StageRow rows_b[4] = {{k + row0 * D, rs, 0, D / 4}, {dout + row0 * D + jb * BV, rs, 2 * D, ncol / 4},
                                {resid + row0 * D + jb * BV, rs, 2 * D + BV, ncol / 4},
                                {dv + row0 * D + jb * BV, rs, 2 * D + 2 * BV, ncol / 4}};
#pragma unroll 1
    for (int i = 0; i < NBUF; ++i) {
      if (i < NBLK) stage_block<4>(slot(i), REC, i * TB, T, rows_b, beta + row0, shift_p, H, 2 * D + 3 * BV);
      cp_commit();
    }
    for (int blk = 0; blk < NBLK; ++blk) {
      const int t0 = blk * TB, tn = min(TB, T - t0);
      cp_wait<NBUF - 1>();
      __syncthreads();
      const float* sl = slot(blk);
      for (int tt = 0; tt < tn; ++tt) {
        const float* rec = sl + tt * REC;
        float kk[NI], gg[CPW], rr[CPW], dr[CPW];
#pragma unroll
        for (int m = 0; m < NI; ++m) {
          const int ii = lane + 32 * m;
          kk[m] = ii < D ? rec[ii] : 0.f;
        }
#pragma unroll
        for (int c = 0; c < CPW; ++c) {
          const bool ok = j0 + c < D;
          gg[c] = ok ? rec[2 * D + warp * CPW + c] : 0.f;
          rr[c] = ok ? rec[2 * D + BV + warp * CPW + c] : 0.f;
          dr[c] = ok ? rec[2 * D + 2 * BV + warp * CPW + c] : 0.f;
        }
        const float bt = staged_beta(rec + 2 * D + 3 * BV, logit, shift_p != nullptr);
#pragma unroll
        for (int m = 0; m < NI; ++m) {
          float a = 0.f;
#pragma unroll
          for (int c = 0; c < CPW; ++c) a = fmaf(S[m][c], dr[c], a);
          const int ii = lane + 32 * m;
          if (ii < D) buf[(tt * NWARP + warp) * D + ii] = a;
        }
#pragma unroll
        for (int m = 0; m < NI; ++m) {
          const float bk = bt * kk[m];
#pragma unroll
          for (int c = 0; c < CPW; ++c) S[m][c] = fmaf(bk, rr[c], S[m][c]);
        }
#pragma unroll
        for (int m = 0; m < NI; ++m) {
          float a = 0.f;
#pragma unroll
          for (int c = 0; c < CPW; ++c) a = fmaf(S[m][c], gg[c], a);
          const int ii = lane + 32 * m;
          if (ii < D) buf1[(tt * NWARP + warp) * D + ii] = a;
        }
      }
      __syncthreads();
      flush_partials(buf, part_hd, row0, H, t0, tn, D);
      flush_partials(buf1, part_dq, row0, H, t0, tn, D);
      if (blk + NBUF < NBLK) stage_block<4>(slot(blk), REC, (blk + NBUF) * TB, T, rows_b, beta + row0, shift_p, H, 2 * D + 3 * BV);
      cp_commit();
      __syncthreads();
    }
    cp_wait<0>();
  }
}

size_t fwd_staged_smem(int D) { return sizeof(float) * (size_t)NBUF * TB * (2 * D + BV + 4); }
size_t bwd_staged_smem(int D) {
  return sizeof(float) * ((size_t)NBUF * TB * (2 * D + 3 * BV + 4) + 2 * (size_t)TB * NWARP * D);
}

// ---- the one-token step (decode) -------------------------------------------------------------
// One CTA of 256 threads per (batch, head): thread t owns the 4-column group j4 = t % (D/4) of
// rows i = t / (D/4) + s * NS (NS = 256 / (D/4) row slices), so every state access is a coalesced
// float4. Pass 1 forms a = H^T k and c = H^T q (partials per slice, summed in slice order through
// shared memory); then r = v - a, o = c + beta (k.q) r (= H'^T q for H' = H + beta k r^T), and
// pass 2 writes H' (the second read of H comes from L2). D a multiple of 4, at most 256.
constexpr int ST = 256;

template <typename E>
__global__ void __launch_bounds__(ST) delta_step_kernel(const E* __restrict__ q, const E* __restrict__ k,
                                                        const E* __restrict__ v, const E* __restrict__ beta,
                                                        const float* __restrict__ shift, int logit, const float* s0,
                                                        float* sn, E* __restrict__ o, int H, int D) {
  __shared__ float ks[256], qs[256], red[2][ST * 4];
  const int bh = blockIdx.x, b = bh / H, tid = threadIdx.x;
  const int quads = D / 4, NS = ST / quads, j4 = tid % quads, slice = tid / quads;
  const int64_t row = bh;  // token row (b * 1 + 0) * H + h
  for (int i = tid; i < D; i += ST) {
    ks[i] = ld_in(k + row * D + i);
    qs[i] = ld_in(q + row * D + i);
  }
  __syncthreads();
  const float* S = s0 + (int64_t)bh * D * D;
  float a[4] = {0.f, 0.f, 0.f, 0.f}, c[4] = {0.f, 0.f, 0.f, 0.f};
  if (slice < NS) {
    for (int i = slice; i < D; i += NS) {
      const float4 w = *reinterpret_cast<const float4*>(S + (int64_t)i * D + 4 * j4);
      const float ki = ks[i], qi = qs[i];
      a[0] = fmaf(w.x, ki, a[0]); a[1] = fmaf(w.y, ki, a[1]); a[2] = fmaf(w.z, ki, a[2]); a[3] = fmaf(w.w, ki, a[3]);
      c[0] = fmaf(w.x, qi, c[0]); c[1] = fmaf(w.y, qi, c[1]); c[2] = fmaf(w.z, qi, c[2]); c[3] = fmaf(w.w, qi, c[3]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      red[0][slice * D + 4 * j4 + e] = a[e];
      red[1][slice * D + 4 * j4 + e] = c[e];
    }
  }
  float kq = 0.f;  // k . q, every thread the same fixed-order sum
  for (int i = 0; i < D; ++i) kq = fmaf(ks[i], qs[i], kq);
  __syncthreads();
  const float bt = beta_at(beta, shift, logit, row, (int64_t)b);
  // r and o for this thread's 4 columns (every slice holds them; slice 0 writes o)
  float r[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int j = 4 * j4 + e;
    float aj = 0.f, cj = 0.f;
    for (int t = 0; t < NS; ++t) {
      aj += red[0][t * D + j];
      cj += red[1][t * D + j];
    }
    r[e] = ld_in(v + row * D + j) - aj;
    if (slice == 0) st_out(o + row * D + j, fmaf(bt * kq, r[e], cj));
  }
  if (slice < NS) {
    float* Sn = sn + (int64_t)bh * D * D;
    for (int i = slice; i < D; i += NS) {
      float4 w = *reinterpret_cast<const float4*>(S + (int64_t)i * D + 4 * j4);
      const float bk = bt * ks[i];
      w.x = fmaf(bk, r[0], w.x); w.y = fmaf(bk, r[1], w.y); w.z = fmaf(bk, r[2], w.z); w.w = fmaf(bk, r[3], w.w);
      *reinterpret_cast<float4*>(Sn + (int64_t)i * D + 4 * j4) = w;
    }
  }
}

int njb(int D) { return (D + BV - 1) / BV; }

int check(int B, int T, int H, int D) {
  VB_REQUIRE(B >= 0 && T >= 0 && H >= 0 && D > 0, "delta_scan_f32: bad shape B=%d T=%d H=%d D=%d", B, T, H, D);
  VB_REQUIRE(D <= 256, "delta_scan_f32: head dimension %d exceeds the kernel's 256", D);
  VB_REQUIRE((int64_t)B * H <= 65535, "delta_scan_f32: B*H = %lld exceeds 65535", (long long)B * H);
  return VB_OK;
}

#define VB_NI_DISPATCH(D, NI, ...)                                    \
  [&]() -> int {                                                      \
    if ((D) <= 32) { constexpr int NI = 1; return __VA_ARGS__(); }    \
    if ((D) <= 64) { constexpr int NI = 2; return __VA_ARGS__(); }    \
    if ((D) <= 128) { constexpr int NI = 4; return __VA_ARGS__(); }   \
    { constexpr int NI = 8; return __VA_ARGS__(); }                   \
  }()

}  // namespace
}  // namespace vb

using namespace vb;

namespace {
int scan_f32_fwd(const float* q, const float* k, const float* v, const float* beta, const float* shift, int logit,
                 const float* state0, float* o, float* state_n, float* resid, int B, int T, int H, int D,
                 void* stream) {
  int rc = check(B, T, H, D);
  if (rc) return rc;
  if (B == 0 || H == 0) return VB_OK;
  VB_REQUIRE(q && k && v && beta && state0 && o && state_n, "delta_scan_f32_fwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid(njb(D), B * H);
  const bool staged = D % 4 == 0 && aligned16(q) && aligned16(k) && aligned16(v);
  return VB_NI_DISPATCH(D, NI, [&]() -> int {
    if (staged && D == 32 * NI) {  // rows in 8 groups of D / 8 (D a power of two from 32 to 256)
      const size_t smem = fwd_staged_smem(D);
      constexpr int R = 4 * NI;
      VB_CUDA_CHECK(cudaFuncSetAttribute(scan_f32_fwd_group_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem), "delta_scan_f32_fwd attr");
      scan_f32_fwd_group_kernel<R><<<grid, NWARP * 32, smem, st>>>(q, k, v, beta, shift, logit, state0, o, state_n,
                                                                   resid, T, H, D);
    } else if (staged) {
      const size_t smem = fwd_staged_smem(D);
      VB_CUDA_CHECK(cudaFuncSetAttribute(scan_f32_fwd_staged_kernel<NI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem), "delta_scan_f32_fwd attr");
      scan_f32_fwd_staged_kernel<NI><<<grid, NWARP * 32, smem, st>>>(q, k, v, beta, shift, logit, state0, o, state_n,
                                                                     resid, T, H, D);
    } else {
      scan_f32_fwd_kernel<NI, float><<<grid, NWARP * 32, 0, st>>>(q, k, v, beta, shift, logit, state0, o, state_n,
                                                                  resid, T, H, D);
    }
    VB_LAUNCH_CHECK("delta_scan_f32_fwd");
    return VB_OK;
  });
}

}  // namespace

extern "C" int vb_delta_scan_f32_fwd(const float* q, const float* k, const float* v, const float* beta,
                                     const float* state0, float* o, float* state_n, float* resid,
                                     int B, int T, int H, int D, void* stream) {
  return scan_f32_fwd(q, k, v, beta, nullptr, 0, state0, o, state_n, resid, B, T, H, D, stream);
}

extern "C" int vb_delta_scan_f32_fwd_logits(const float* q, const float* k, const float* v,
                                            const float* beta_logits, const float* shift, const float* state0,
                                            float* o, float* state_n, float* resid, int B, int T, int H, int D,
                                            void* stream) {
  return scan_f32_fwd(q, k, v, beta_logits, shift, 1, state0, o, state_n, resid, B, T, H, D, stream);
}

extern "C" int vb_delta_scan_step(const void* q, const void* k, const void* v, const void* beta,
                                  const float* shift, int from_logits, const float* state0, float* state_n, void* o,
                                  int B, int H, int D, int dtype, void* stream) {
  int rc = check(B, 1, H, D);
  if (rc) return rc;
  if (B == 0 || H == 0) return VB_OK;
  VB_REQUIRE(D % 4 == 0, "delta_scan_step: head dimension %d must be a multiple of 4", D);
  VB_REQUIRE(q && k && v && beta && state0 && state_n && o, "delta_scan_step: null pointer");
  VB_REQUIRE(aligned16(state0) && aligned16(state_n), "delta_scan_step: state not 16-byte aligned");
  VB_REQUIRE(dtype == VB_F32 || dtype == VB_BF16, "delta_scan_step: dtype must be float32 or bfloat16");
  cudaStream_t st = (cudaStream_t)stream;
  const int logit = from_logits ? 1 : 0;
  const unsigned grid = (unsigned)(B * H);
  if (dtype == VB_F32) {
    delta_step_kernel<float><<<grid, ST, 0, st>>>((const float*)q, (const float*)k, (const float*)v,
                                                  (const float*)beta, shift, logit, state0, state_n, (float*)o, H, D);
  } else {
    using bf = __nv_bfloat16;
    delta_step_kernel<bf><<<grid, ST, 0, st>>>((const bf*)q, (const bf*)k, (const bf*)v, (const bf*)beta, shift,
                                               logit, state0, state_n, (bf*)o, H, D);
  }
  VB_LAUNCH_CHECK("delta_scan_step");
  return VB_OK;
}

extern "C" size_t vb_delta_scan_f32_bwd_workspace(int B, int T, int H, int D) {
  const size_t rows = (size_t)(B > 0 ? B : 0) * (size_t)(T > 0 ? T : 0) * (size_t)(H > 0 ? H : 0);
  return 3 * (size_t)njb(D > 0 ? D : 1) * (rows > 0 ? rows : 1) * (size_t)(D > 0 ? D : 1) * sizeof(float);
}

namespace {
int scan_f32_bwd(const float* q, const float* k, const float* beta, const float* shift, int logit,
                 const float* state0, const float* resid, const float* dout, const float* dstate_n, float* dq,
                 float* dk, float* dv, float* dbeta, float* dstate0, void* workspace, int B, int T, int H, int D,
                 void* stream) {
  int rc = check(B, T, H, D);
  if (rc) return rc;
  if (B == 0 || H == 0) return VB_OK;
  VB_REQUIRE(q && k && beta && state0 && resid && dout && dq && dk && dv && dbeta && dstate0 && workspace,
             "delta_scan_f32_bwd: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid(njb(D), B * H);
  const size_t smem = sizeof(float) * NWARP * D;
  float* part = (float*)workspace;
  const bool staged = D % 4 == 0 && aligned16(q) && aligned16(k) && aligned16(resid) && aligned16(dout) &&
                      aligned16(dv);
  return VB_NI_DISPATCH(D, NI, [&]() -> int {
    if (staged) {
      const size_t sm = bwd_staged_smem(D);
      if (D == 32 * NI) {
        VB_CUDA_CHECK(cudaFuncSetAttribute(scan_f32_bwd_staged_kernel<NI, true>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm), "delta_scan_f32_bwd attr");
        scan_f32_bwd_staged_kernel<NI, true><<<grid, NWARP * 32, sm, st>>>(q, k, beta, shift, logit, state0, resid,
                                                                           dout, dstate_n, dv, dstate0, part, B, T, H, D);
      } else {
        VB_CUDA_CHECK(cudaFuncSetAttribute(scan_f32_bwd_staged_kernel<NI, false>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm), "delta_scan_f32_bwd attr");
        scan_f32_bwd_staged_kernel<NI, false><<<grid, NWARP * 32, sm, st>>>(q, k, beta, shift, logit, state0, resid,
                                                                            dout, dstate_n, dv, dstate0, part, B, T, H, D);
      }
    } else {
      scan_f32_bwd_kernel<NI><<<grid, NWARP * 32, smem, st>>>(q, k, beta, shift, logit, state0, resid, dout,
                                                              dstate_n, dv, dstate0, part, B, T, H, D);
    }
    VB_LAUNCH_CHECK("delta_scan_f32_bwd");
    const int64_t rows = (int64_t)B * T * H;
    if (rows > 0) {
      scan_f32_finish_kernel<<<(int)((rows + 7) / 8), 256, 0, st>>>(k, beta, shift, logit, part, dq, dk, dbeta,
                                                                    rows, H, D, njb(D));
      VB_LAUNCH_CHECK("delta_scan_f32_finish");
    }
    return VB_OK;
  });
}
}  // namespace

extern "C" int vb_delta_scan_f32_bwd(const float* q, const float* k, const float* v, const float* beta,
                                     const float* state0, const float* resid, const float* dout,
                                     const float* dstate_n, float* dq, float* dk, float* dv,
                                     float* dbeta, float* dstate0, void* workspace, int B, int T,
                                     int H, int D, void* stream) {
  (void)v;
  return scan_f32_bwd(q, k, beta, nullptr, 0, state0, resid, dout, dstate_n, dq, dk, dv, dbeta, dstate0,
                      workspace, B, T, H, D, stream);
}

extern "C" int vb_delta_scan_f32_bwd_logits(const float* q, const float* k, const float* v,
                                            const float* beta_logits, const float* shift, const float* state0,
                                            const float* resid, const float* dout, const float* dstate_n, float* dq,
                                            float* dk, float* dv, float* dlogits, float* dstate0, void* workspace,
                                            int B, int T, int H, int D, void* stream) {
  (void)v;
  return scan_f32_bwd(q, k, beta_logits, shift, 1, state0, resid, dout, dstate_n, dq, dk, dv, dlogits, dstate0,
                      workspace, B, T, H, D, stream);
}
