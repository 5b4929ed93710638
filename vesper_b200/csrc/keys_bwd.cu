// The key filter backward: the launcher, the workspace query and the C entry points (kernels in
// keys.cuh).
#include "keys.cuh"

namespace vb {
namespace {

template <typename T>
int launch_bwd(const void* z, const float* hist, const float* taps, const void* gk, const float* stats, void* dz,
               float* dtaps, float* dhist, float* partial, int B, int T_, int W, int heads, int K, float floor_,
               cudaStream_t st) {
  const int hd = W / heads, epl = epl_bwd(hd);
  const int spans = (W + 32 * epl - 1) / (32 * epl);
  int parts = 0;
  const int rc = VB_EPL_DISPATCH(epl, EPL, [&]() -> int {
    return VB_K_DISPATCH(K, KK, [&]() -> int {
      const int runs = (T_ + run_len(RUN_B, KK) - 1) / run_len(RUN_B, KK);
      parts = B * runs;
      const int64_t warps = (int64_t)B * spans * runs;
      const int ctas = (int)((warps + WARPS - 1) / WARPS);
      const int G = hd / EPL;
      auto go = [&](auto gt) {
        constexpr int GG = decltype(gt)::value;
        if (stats != nullptr)
          keys_bwd_kernel<T, EPL, KK, true, GG><<<ctas, WARPS * 32, 0, st>>>(
              (const T*)z, hist, taps, (const T*)gk, (const float2*)stats, (T*)dz, dhist, partial, B, T_, W, hd, spans,
              runs, floor_);
        else
          keys_bwd_kernel<T, EPL, KK, false, GG><<<ctas, WARPS * 32, 0, st>>>(
              (const T*)z, hist, taps, (const T*)gk, nullptr, (T*)dz, dhist, partial, B, T_, W, hd, spans, runs,
              floor_);
      };
      if constexpr (KK == 4 && EPL == 4) {
        if (G == 32) go(std::integral_constant<int, 32>{});
        else if (G == 16) go(std::integral_constant<int, 16>{});
        else go(std::integral_constant<int, 0>{});
      } else {
        go(std::integral_constant<int, 0>{});
      }
      VB_LAUNCH_CHECK("keys_bwd");
      return VB_OK;
    });
  });
  if (rc) return rc;
  return column_sum(partial, dtaps, parts, K * W, st);
}

}  // namespace
}  // namespace vb

using namespace vb;

extern "C" size_t vb_keys_bwd_workspace(int B, int T, int width, int heads, int taps_count) {
  // runs of at least RUN_B tokens: never more partial rows than ceil(T / RUN_B) per batch row
  const int runs = (T + RUN_B - 1) / RUN_B;
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
  VB_REQUIRE(aligned16(workspace) && (!grad_hist || aligned16(grad_hist)),
             "keys_bwd: the workspace and the history gradient must start on 16-byte boundaries");
  return VB_DISPATCH_DTYPE(dtype, Tt, [&]() -> int {
    return launch_bwd<Tt>(z, hist, taps, grad_keys, stats, grad_z, grad_taps, grad_hist, (float*)workspace, B, T,
                          width, heads, taps_count, floor_, st);
  });
}
