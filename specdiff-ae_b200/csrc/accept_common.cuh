// Device helpers shared by the acceptance scan (accept.cu) and the fused
// lm_head + acceptance kernel (lmhead.cu): the torch.argmax comparison and
// the Gumbel noise of sampled acceptance.
#pragma once

#include "common.cuh"

namespace tv {
namespace acc {

struct Best {
  float v;
  int i;
};

__device__ __forceinline__ bool better(float v1, int i1, float v2, int i2) {
  const bool n1 = v1 != v1, n2 = v2 != v2;
  if (n1 || n2) return n1 && (!n2 || i1 < i2);
  return v1 > v2 || (v1 == v2 && i1 < i2);
}

__device__ __forceinline__ void take(Best& b, float v, int i) {
  if (better(v, i, b.v, b.i)) { b.v = v; b.i = i; }
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as
// easy as 1, 2, 3", SC'11): 10 rounds of two 32x32->64 multiplies with
// Weyl-sequence key bumps.
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += W0;
    k.y += W1;
  }
  return c;
}

// Gumbel(0, 1) noise for (row, token j) from a 24-bit uniform in (0, 1).
__device__ __forceinline__ float gumbel(uint64_t seed, uint64_t offset, int row, int j) {
  const uint4 r = philox4x32_10(make_uint4((uint32_t)(j >> 2), (uint32_t)row, (uint32_t)offset,
                                           (uint32_t)(offset >> 32)),
                                make_uint2((uint32_t)seed, (uint32_t)(seed >> 32)));
  const uint32_t w = (j & 3) == 0 ? r.x : (j & 3) == 1 ? r.y : (j & 3) == 2 ? r.z : r.w;
  const float u = ((float)(w >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

}  // namespace acc

// Stage 2 of the acceptance: per-node argmax over `chunks` (score, index)
// partials per row ([rows][chunks]), or the given `sampled` tokens, then the
// acceptance rule, path and result block of tv_accept.  With draft == NULL
// only next_tokens is written.  A nonzero *upstream_err (the stage that
// produced the partials gave up on a wait) makes every next token -1 and
// result[0] TV_ERR_LAUNCH instead.
int launch_accept_decide(int rows, int chunks, const float* part_v, const int* part_i, const int64_t* sampled,
                         const int64_t* draft, const int64_t* parent, const int64_t* pos, int max_depth,
                         int64_t* next_tokens, int64_t* result, const int* upstream_err, cudaStream_t st);

}  // namespace tv
