// TMA tensor maps of the library's tensors.
#pragma once
#include <cuda.h>

namespace vb {
// A 4-D map over a bf16 (or, with f16 set, float16) [B, T, H, D] array: boxes of 64 channels x 1 head x 64 tokens x 1 row,
// 128-byte swizzle (the tiles' shared-memory layout), zero fill outside the array (past T, past D).
int make_token_map(CUtensorMap* map, const void* base, int B, int T, int H, int D, bool f16 = false);
}  // namespace vb
