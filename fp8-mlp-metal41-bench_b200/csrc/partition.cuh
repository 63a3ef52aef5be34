// partition.cuh -- stream-K partition of U work units over G persistent CTAs.
//
// CTA c takes the contiguous run [c*U/G, (c+1)*U/G): runs differ in length by
// at most one unit, and a unit's owner follows from its index alone, so every
// CTA can name the other contributors to a shared output tile without
// communicating.
#pragma once
#include <cuda_runtime.h>

namespace mlpg {

// contiguous unit range of CTA c of G
__device__ __forceinline__ void cta_range(int c, int G, int U, int& u0, int& u1) {
  u0 = (int)((long long)c * U / G);
  u1 = (int)((long long)(c + 1) * U / G);
}

// the CTA whose (non-empty) range contains unit u
__device__ __forceinline__ int owner_of(int u, int G, int U) {
  int c = (int)(((long long)u * G + G - 1) / U);   // largest c with c*U/G <= u
  while (c > 0 && (long long)c * U / G > u) --c;
  while ((long long)(c + 1) * U / G <= u) ++c;
  return c;
}

}  // namespace mlpg
