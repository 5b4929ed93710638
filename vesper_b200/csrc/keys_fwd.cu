// The key filter forward: the launcher and the C entry point (kernels in keys.cuh).
#include "keys.cuh"

namespace vb {
namespace {

template <typename T>
int launch_fwd(const void* z, const float* hist, const float* taps, void* out, float* stats, int B, int T_, int W,
               int heads, int K, float floor_, cudaStream_t st) {
  const int hd = W / heads;
  const int epl = epl_fwd<T>(hd);
  const int spans = (W + 32 * epl - 1) / (32 * epl);
  return VB_EPL_DISPATCH(epl, EPL, [&]() -> int {
    return VB_K_DISPATCH(K, KK, [&]() -> int {
      const int runs = (T_ + run_len(RUN_F, KK) - 1) / run_len(RUN_F, KK);
      const int64_t warps = (int64_t)B * spans * runs;
      const int ctas = (int)((warps + WARPS - 1) / WARPS);
      const int G = hd / EPL;
      auto go = [&](auto gt) {
        keys_fwd_kernel<T, EPL, KK, decltype(gt)::value><<<ctas, WARPS * 32, 0, st>>>(
            (const T*)z, hist, taps, (T*)out, (float2*)stats, B, T_, W, hd, spans, runs, floor_);
      };
      // the filter width and head layouts in use get the lanes per head as a constant
      if constexpr (KK == 4 && EPL == 16 / (int)sizeof(T)) {
        if (G == 16) go(std::integral_constant<int, 16>{});
        else if (G == 8) go(std::integral_constant<int, 8>{});
        else if (G == 32) go(std::integral_constant<int, 32>{});
        else go(std::integral_constant<int, 0>{});
      } else {
        go(std::integral_constant<int, 0>{});
      }
      VB_LAUNCH_CHECK("keys_fwd");
      return VB_OK;
    });
  });
}

}  // namespace
}  // namespace vb

using namespace vb;

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
  cudaStream_t st = (cudaStream_t)stream;
  return VB_DISPATCH_DTYPE(dtype, Tt, [&]() -> int {
    return launch_fwd<Tt>(z, hist, taps, keys, stats, B, T, width, heads, taps_count, floor_, st);
  });
}
