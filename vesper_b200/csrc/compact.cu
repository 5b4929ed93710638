// The loop's active-token bookkeeping: compaction of the active set, and the row copies that move
// per-token rows between the dense [B, N] layout and compact buffers, or merge fresh rows with
// carried ones (copy-forward). Byte work, HBM-bound: 16-byte vector copies where rows allow.
//
// Replaces, for mstampfli/vesper-preview's loop (vesper/loop.py:349-465, :523-537) and column
// (vesper/column.py:140-143, :779-796), the per-tensor torch.where merges and the dense compute of
// halted tokens: one launch moves every tensor of a merge, and a compact index list lets the
// attention compute only the active queries.
//
// compact_index: one CTA per batch row, a block-wide prefix count over `active` in 1024-token tiles:
//   idx[b][r]  = t for the r-th active token t (r < count), -1 beyond (padding);
//   rank[b][t] = r for an active token, -1 for a halted one;  counts[b] = the active count;
//   qpos[b][r] = idx + qpos_offset (optional; the attention's key index of a compact row).
// Row copies: up to 12 tensors per launch, each a [B, rows, row_bytes] byte array; an
// index outside its range, or a null source, yields zero bytes (never an out-of-range read).
#include "common.cuh"

namespace vb {
namespace {

constexpr int MAXT = 12;  // tensors per copy launch

struct RowSets {
  const uint8_t* a[MAXT];  // first source (fresh / compact) or null = zeros
  const uint8_t* b[MAXT];  // second source (carried / fallback) or null = zeros
  uint8_t* out[MAXT];
  int64_t row_bytes[MAXT];
  int vec[MAXT];    // copy unit in bytes: 16, 4 or 1 (every pointer and row_bytes a multiple)
  int lshift[MAXT];  // log2 of the lanes that copy one row: enough for its units, at most 32
  int n;
};

// Tensor i of a launch is blockIdx.y; its rows go to teams of 2^lshift lanes (a row of 16 bytes
// takes one lane, a row of 512 bytes or more a warp), the teams striding over the rows.
struct Team {
  int64_t first, stride;  // this team's first row, the number of teams
  int lane, size;         // lane within the team, lanes per team
};

__device__ __forceinline__ Team team_of(const RowSets& s, int i) {
  const int sh = s.lshift[i];
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> sh;
  return Team{t, ((int64_t)gridDim.x * blockDim.x) >> sh, (int)(threadIdx.x & ((1u << sh) - 1u)), 1 << sh};
}

template <int U>
__device__ __forceinline__ void copy_unit(uint8_t* dst, const uint8_t* src, int64_t off) {
  if constexpr (U == 16) {
    *reinterpret_cast<uint4*>(dst + off) = src ? *reinterpret_cast<const uint4*>(src + off) : make_uint4(0, 0, 0, 0);
  } else if constexpr (U == 4) {
    *reinterpret_cast<uint32_t*>(dst + off) = src ? *reinterpret_cast<const uint32_t*>(src + off) : 0u;
  } else {
    dst[off] = src ? src[off] : (uint8_t)0;
  }
}

// Copies row `row_out` of tensor i from `src_row` of `src` (null = zeros); the team's lanes stride
// the row in copy units.
__device__ __forceinline__ void copy_row(const RowSets& s, int i, const uint8_t* src, int64_t src_row, int64_t row_out,
                                         const Team& tm) {
  const int64_t rb = s.row_bytes[i];
  uint8_t* dst = s.out[i] + row_out * rb;
  const uint8_t* sp = src ? src + src_row * rb : nullptr;
  const int u = s.vec[i];
  if (u == 16) {
    for (int64_t off = (int64_t)tm.lane * 16; off < rb; off += tm.size * 16) copy_unit<16>(dst, sp, off);
  } else if (u == 4) {
    for (int64_t off = (int64_t)tm.lane * 4; off < rb; off += tm.size * 4) copy_unit<4>(dst, sp, off);
  } else {
    for (int64_t off = tm.lane; off < rb; off += tm.size) copy_unit<1>(dst, sp, off);
  }
}

// out[t] = (mask[t] != invert) ? a[t] : b[t]
__global__ void select_rows_kernel(const uint8_t* __restrict__ mask, int invert, RowSets s, int64_t tokens) {
  const int i = blockIdx.y;
  const Team tm = team_of(s, i);
  for (int64_t t = tm.first; t < tokens; t += tm.stride) {
    const bool pick_a = (mask[t] != 0) != (invert != 0);
    copy_row(s, i, pick_a ? s.a[i] : s.b[i], t, t, tm);
  }
}

// out[b][r] = r < counts[b] and 0 <= idx[b][r] < N ? a[b][idx] : 0       (compact <- dense)
__global__ void gather_rows_kernel(const int* __restrict__ idx, const int* __restrict__ counts, RowSets s, int B,
                                   int N, int NC) {
  const int i = blockIdx.y;
  const Team tm = team_of(s, i);
  const int64_t rows = (int64_t)B * NC;  // below 2^31 (checked by the entry point)
  for (int64_t br = tm.first; br < rows; br += tm.stride) {
    const int b = (int)br / NC, r = (int)br - b * NC;
    const int c = counts ? counts[b] : NC;
    const int t = r < c ? idx[br] : -1;
    const bool ok = t >= 0 && t < N;
    copy_row(s, i, ok ? s.a[i] : nullptr, (int64_t)b * N + (ok ? t : 0), br, tm);
  }
}

// out[b][t] = 0 <= rank[b][t] < NC ? a[b][rank] : b_src[b][t]             (dense <- compact)
__global__ void expand_rows_kernel(const int* __restrict__ rank, RowSets s, int B, int N, int NC) {
  const int i = blockIdx.y;
  const Team tm = team_of(s, i);
  const int64_t rows = (int64_t)B * N;  // below 2^31 (checked by the entry point)
  for (int64_t bt = tm.first; bt < rows; bt += tm.stride) {
    const int b = (int)bt / N;
    const int r = rank[bt];
    if (r >= 0 && r < NC) copy_row(s, i, s.a[i], (int64_t)b * NC + r, bt, tm);
    else copy_row(s, i, s.b[i], bt, bt, tm);
  }
}

// The end of the bucket that runs for `c` active rows: the smallest first * 2^k >= c, clamped to
// the buffer's NC rows (0 when no row is active).
__device__ __forceinline__ int slab_end(int c, int first, int NC) {
  if (c <= 0) return 0;
  long long end = first;
  while (end < c) end *= 2;
  return (int)(end < NC ? end : NC);
}

// As gather_rows_kernel, for compact buffers that bucketed work reads: rows from counts[b] to the
// end of the bucket are zeroed, the rows past it are left as they are (never read). Tensor i is
// blockIdx.y; the warps stride over the rows that are written only (no per-row index division).
__global__ void gather_slabs_kernel(const int* __restrict__ idx, const int* __restrict__ counts, RowSets s, int B,
                                    int N, int NC, int first) {
  const int i = blockIdx.y;
  const Team tm = team_of(s, i);
  for (int b = 0; b < B; ++b) {
    const int c = counts[b];
    const int end = slab_end(c, first, NC);
    for (int64_t r = tm.first; r < end; r += tm.stride) {
      const int64_t br = (int64_t)b * NC + r;
      const int t = r < c ? idx[br] : -1;
      const bool ok = t >= 0 && t < N;
      copy_row(s, i, ok ? s.a[i] : nullptr, (int64_t)b * N + (ok ? t : 0), br, tm);
    }
  }
}

// One compaction of all B x N tokens from the per-row one: base = the active tokens of the rows
// before b; flat_idx[base + r] = b N + idx[b][r] (r < counts[b]), flat_rank[b N + t] = base +
// rank[b][t] (or -1), *flat_count = the total. Optionally the map between the flat compact rows and
// the per-row compact rows (b, r) at b N + r: flat_pb[base + r] = b N + r, pb_flat[b N + r] = base + r
// (r < counts[b], else -1). One CTA per row; the base is a sum over counts.
constexpr int FLAT_T = 256;
__global__ void __launch_bounds__(FLAT_T) flatten_compaction_kernel(const int* __restrict__ idx,
                                                                    const int* __restrict__ rank,
                                                                    const int* __restrict__ counts, int B, int N,
                                                                    int* __restrict__ flat_idx,
                                                                    int* __restrict__ flat_rank,
                                                                    int* __restrict__ flat_count,
                                                                    int* __restrict__ flat_pb,
                                                                    int* __restrict__ pb_flat) {
  __shared__ int part[FLAT_T / 32];
  const int b = blockIdx.x, tid = threadIdx.x;
  int before = 0, all = 0;
  for (int j = tid; j < B; j += FLAT_T) {
    const int c = counts[j];
    all += c;
    if (j < b) before += c;
  }
  before = __reduce_add_sync(0xffffffffu, before);
  if ((tid & 31) == 0) part[tid >> 5] = before;
  __syncthreads();
  int base = 0;
#pragma unroll
  for (int w = 0; w < FLAT_T / 32; ++w) base += part[w];
  if (b == 0) {
    __syncthreads();
    all = __reduce_add_sync(0xffffffffu, all);
    if ((tid & 31) == 0) part[tid >> 5] = all;
    __syncthreads();
    if (tid == 0) {
      int total = 0;
      for (int w = 0; w < FLAT_T / 32; ++w) total += part[w];
      *flat_count = total;
    }
  }
  const int c = counts[b];
  const int64_t row = (int64_t)b * N;
  for (int r = tid; r < c; r += FLAT_T) flat_idx[base + r] = (int)(row + idx[row + r]);
  for (int t = tid; t < N; t += FLAT_T) {
    const int k = rank[row + t];
    flat_rank[row + t] = k >= 0 ? base + k : -1;
  }
  if (flat_pb != nullptr && pb_flat != nullptr) {
    for (int r = tid; r < c; r += FLAT_T) flat_pb[base + r] = (int)(row + r);
    for (int r = tid; r < N; r += FLAT_T) pb_flat[row + r] = r < c ? base + r : -1;
  }
}

constexpr int SCAN_T = 1024;

__global__ void __launch_bounds__(SCAN_T) compact_index_kernel(const uint8_t* __restrict__ active, int* __restrict__ idx,
                                                               int* __restrict__ rank, int* __restrict__ counts,
                                                               int* __restrict__ qpos, int N, int qpos_offset) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint8_t* act = active + (int64_t)b * N;
  if (tid == 0) base_s = 0;
  __syncthreads();
  for (int t0 = 0; t0 < N; t0 += SCAN_T) {
    const int t = t0 + tid;
    const int a = (t < N && act[t]) ? 1 : 0;
    const unsigned bal = __ballot_sync(0xffffffffu, a);
    const int in_warp = __popc(bal & ((1u << lane) - 1u));
    if (lane == 0) warp_tot[warp] = __popc(bal);
    __syncthreads();
    if (warp == 0) {
      const int v = warp_tot[lane];
      int inc = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      warp_tot[lane] = inc - v;  // exclusive prefix of the warps
    }
    __syncthreads();
    const int base = base_s;
    const int r = base + warp_tot[warp] + in_warp;
    if (t < N) {
      rank[(int64_t)b * N + t] = a ? r : -1;
      if (a) {
        idx[(int64_t)b * N + r] = t;
        if (qpos) qpos[(int64_t)b * N + r] = t + qpos_offset;
      }
    }
    __syncthreads();
    if (tid == SCAN_T - 1) base_s = r + a;  // the last thread's inclusive total
    __syncthreads();
  }
  const int total = base_s;
  for (int r = total + tid; r < N; r += SCAN_T) {
    idx[(int64_t)b * N + r] = -1;
    if (qpos) qpos[(int64_t)b * N + r] = -1;
  }
  if (tid == 0) counts[b] = total;
}

int fill_sets(RowSets& s, int n, const void* const* a, const void* const* b, void* const* out,
              const long long* row_bytes, const char* what) {
  VB_REQUIRE(n >= 1 && n <= MAXT, "%s: %d tensors, at most %d per call", what, n, MAXT);
  VB_REQUIRE(out && row_bytes, "%s: null array", what);
  s.n = n;
  for (int i = 0; i < n; ++i) {
    VB_REQUIRE(out[i] != nullptr && row_bytes[i] > 0, "%s: tensor %d has no output or an empty row", what, i);
    s.a[i] = a ? (const uint8_t*)a[i] : nullptr;
    s.b[i] = b ? (const uint8_t*)b[i] : nullptr;
    s.out[i] = (uint8_t*)out[i];
    s.row_bytes[i] = row_bytes[i];
    auto all = [&](uintptr_t m) {
      return ((uintptr_t)s.out[i] & m) == 0 && ((uintptr_t)s.a[i] & m) == 0 && ((uintptr_t)s.b[i] & m) == 0 &&
             ((uint64_t)row_bytes[i] & m) == 0;
    };
    s.vec[i] = all(15) ? 16 : all(3) ? 4 : 1;
    const int64_t units = row_bytes[i] / s.vec[i];
    int sh = 0;
    while (sh < 5 && ((int64_t)1 << sh) < units) ++sh;
    s.lshift[i] = sh;
  }
  return VB_OK;
}

// The launch of a row-copy kernel over `rows` rows of each tensor: blocks of 256 threads, enough
// for every row's team where the widest team decides, at most 8 blocks per SM (the teams then
// stride), one grid row per tensor.
dim3 grid_rows(const RowSets& s, int64_t rows) {
  int sh = 0;
  for (int i = 0; i < s.n; ++i) sh = s.lshift[i] > sh ? s.lshift[i] : sh;
  const int64_t blocks = (rows * ((int64_t)1 << sh) + 255) / 256;
  const int64_t cap = 148 * 8;
  return dim3((unsigned)(blocks < 1 ? 1 : blocks < cap ? blocks : cap), (unsigned)s.n);
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" int vb_compact_index(const unsigned char* active, int* idx, int* rank, int* counts, int* qpos, int B, int N,
                                int qpos_offset, void* stream) {
  VB_REQUIRE(B >= 0 && N >= 0, "compact_index: bad shape B=%d N=%d", B, N);
  if (B == 0) return VB_OK;
  VB_REQUIRE(active && idx && rank && counts, "compact_index: null pointer");
  compact_index_kernel<<<B, SCAN_T, 0, (cudaStream_t)stream>>>(active, idx, rank, counts, qpos, N, qpos_offset);
  VB_LAUNCH_CHECK("compact_index");
  return VB_OK;
}

extern "C" int vb_select_rows(const unsigned char* mask, int invert, int ntensors, const void* const* a,
                              const void* const* b, void* const* out, const long long* row_bytes, long long tokens,
                              void* stream) {
  VB_REQUIRE(tokens >= 0, "select_rows: negative token count");
  if (tokens == 0) return VB_OK;
  VB_REQUIRE(mask != nullptr, "select_rows: null mask");
  RowSets s;
  int rc = fill_sets(s, ntensors, a, b, out, row_bytes, "select_rows");
  if (rc) return rc;
  select_rows_kernel<<<grid_rows(s, tokens), 256, 0, (cudaStream_t)stream>>>(mask, invert, s, tokens);
  VB_LAUNCH_CHECK("select_rows");
  return VB_OK;
}

extern "C" int vb_gather_rows(const int* idx, const int* counts, int B, int N, int NC, int ntensors,
                              const void* const* src, void* const* dst, const long long* row_bytes, void* stream) {
  VB_REQUIRE(B >= 0 && N >= 0 && NC >= 0, "gather_rows: bad shape B=%d N=%d NC=%d", B, N, NC);
  VB_REQUIRE((int64_t)B * NC <= 0x7fffffff && (int64_t)B * N <= 0x7fffffff, "gather_rows: rows exceed int32 indices");
  if ((int64_t)B * NC == 0) return VB_OK;
  VB_REQUIRE(idx != nullptr, "gather_rows: null index");
  RowSets s;
  int rc = fill_sets(s, ntensors, src, nullptr, dst, row_bytes, "gather_rows");
  if (rc) return rc;
  gather_rows_kernel<<<grid_rows(s, (int64_t)B * NC), 256, 0, (cudaStream_t)stream>>>(idx, counts, s, B, N, NC);
  VB_LAUNCH_CHECK("gather_rows");
  return VB_OK;
}

extern "C" int vb_gather_rows_slabs(const int* idx, const int* counts, int B, int N, int NC, int first, int ntensors,
                                    const void* const* src, void* const* dst, const long long* row_bytes,
                                    void* stream) {
  VB_REQUIRE(B >= 0 && N >= 0 && NC >= 0 && first > 0, "gather_rows_slabs: bad shape B=%d N=%d NC=%d first=%d", B, N,
             NC, first);
  if ((int64_t)B * NC == 0) return VB_OK;
  VB_REQUIRE(idx != nullptr && counts != nullptr, "gather_rows_slabs: null index or counts");
  RowSets s;
  int rc = fill_sets(s, ntensors, src, nullptr, dst, row_bytes, "gather_rows_slabs");
  if (rc) return rc;
  dim3 grid = grid_rows(s, (int64_t)NC);  // teams for one batch row's worth: most return at once
  grid.x = grid.x < 148 * 4 ? grid.x : 148 * 4;
  gather_slabs_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(idx, counts, s, B, N, NC, first);
  VB_LAUNCH_CHECK("gather_rows_slabs");
  return VB_OK;
}

extern "C" int vb_flatten_compaction(const int* idx, const int* rank, const int* counts, int B, int N, int* flat_idx,
                                     int* flat_rank, int* flat_count, int* flat_pb, int* pb_flat, void* stream) {
  VB_REQUIRE(B >= 0 && N >= 0, "flatten_compaction: bad shape B=%d N=%d", B, N);
  VB_REQUIRE((int64_t)B * N <= 0x7fffffff, "flatten_compaction: %lld tokens exceed int32 indices", (long long)B * N);
  if (B == 0) return VB_OK;
  VB_REQUIRE(idx && rank && counts && flat_idx && flat_rank && flat_count, "flatten_compaction: null pointer");
  flatten_compaction_kernel<<<B, FLAT_T, 0, (cudaStream_t)stream>>>(idx, rank, counts, B, N, flat_idx, flat_rank,
                                                                    flat_count, flat_pb, pb_flat);
  VB_LAUNCH_CHECK("flatten_compaction");
  return VB_OK;
}

extern "C" int vb_expand_rows(const int* rank, int B, int N, int NC, int ntensors, const void* const* src,
                              const void* const* fallback, void* const* dst, const long long* row_bytes,
                              void* stream) {
  VB_REQUIRE(B >= 0 && N >= 0 && NC >= 0, "expand_rows: bad shape B=%d N=%d NC=%d", B, N, NC);
  VB_REQUIRE((int64_t)B * N <= 0x7fffffff && (int64_t)B * NC <= 0x7fffffff, "expand_rows: rows exceed int32 indices");
  if ((int64_t)B * N == 0) return VB_OK;
  VB_REQUIRE(rank != nullptr, "expand_rows: null rank");
  RowSets s;
  int rc = fill_sets(s, ntensors, src, fallback, dst, row_bytes, "expand_rows");
  if (rc) return rc;
  expand_rows_kernel<<<grid_rows(s, (int64_t)B * N), 256, 0, (cudaStream_t)stream>>>(rank, s, B, N, NC);
  VB_LAUNCH_CHECK("expand_rows");
  return VB_OK;
}
