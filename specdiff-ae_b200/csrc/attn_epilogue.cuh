// Output epilogues of the verify-attention kernels: final O / LSE / merge
// weight for one query row, or the split-KV partial of one row.
#pragma once

#include "attn_params.cuh"
#include "common.cuh"

namespace tv {

// Query row r of (batch b, kv head hk) -> (node m, query head h).
__device__ __forceinline__ void row_coords(const AttnParams& p, int hk, int r, int& m, int& h) {
  m = r / p.G;
  h = hk * p.G + (r - m * p.G);
}

// Two consecutive head-dim values (d, d+1) of a final output row.
template <typename T>
__device__ __forceinline__ void store_out_pair(const AttnParams& p, int b, int m, int h, int d, float v0, float v1) {
  const int64_t off = (int64_t)b * p.o_sb + (int64_t)m * p.o_sm + (int64_t)h * p.o_sh + d;
  if (p.out_f32) {
    *reinterpret_cast<float2*>(static_cast<float*>(p.out) + off) = make_float2(v0, v1);
  } else {
    *reinterpret_cast<uint32_t*>(static_cast<T*>(p.out) + off) = Elem<T>::pack2(v0, v1);
  }
}

// LSE and the optional merge weight sigmoid(aux_lse - lse) of a final row.
template <typename T>
__device__ __forceinline__ void store_row_stats(const AttnParams& p, int b, int m, int h, float lse) {
  if (p.lse) p.lse[(int64_t)b * p.lse_sb + (int64_t)m * p.lse_sm + (int64_t)h * p.lse_sh] = lse;
  if (p.aux) {
    const float a = p.aux[(int64_t)b * p.aux_sb + (int64_t)m * p.aux_sm + (int64_t)h * p.aux_sh];
    // sigmoid(a - lse) = 1 / (1 + exp(lse - a)); lse = -inf gives 1.
    const float w = 1.0f / (1.0f + expf(lse - a));
    static_cast<T*>(p.weight)[(int64_t)b * p.w_sb + (int64_t)m * p.w_sm + (int64_t)h * p.w_sh] = Elem<T>::from_f(w);
  }
}

__device__ __forceinline__ float* part_o_row(const AttnParams& p, int split, int bh, int r, int D) {
  return p.part_o + (((int64_t)split * p.B * p.Hkv + bh) * p.R + r) * D;
}
__device__ __forceinline__ float* part_lse_row(const AttnParams& p, int split, int bh, int r) {
  return p.part_lse + ((int64_t)split * p.B * p.Hkv + bh) * p.R + r;
}

// Log-sum-exp combine of the p.splits split partials of kernel row (bh, r):
// this thread's four head-dim values 4q .. 4q+3 (normalised) and the row's
// LSE.  Partials are read BLK splits at a time (all loads of a block in
// flight together; they are usually still in L2) and folded with a running
// max, so the row needs one pass.
template <int D, int BLK = 8>
__device__ __forceinline__ void combine_split_row(const AttnParams& p, int bh, int r, int q, float4& o,
                                                  float& lse) {
  float mx = -INFINITY, wsum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s0 = 0; s0 < p.splits; s0 += BLK) {
    float l[BLK];
    float4 v[BLK];
#pragma unroll
    for (int j = 0; j < BLK; ++j) {
      const int s = s0 + j;
      if (s < p.splits) {
        l[j] = *part_lse_row(p, s, bh, r);
        v[j] = *reinterpret_cast<const float4*>(part_o_row(p, s, bh, r, D) + 4 * q);
      } else {
        l[j] = -INFINITY;
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    float bm = l[0];
#pragma unroll
    for (int j = 1; j < BLK; ++j) bm = fmaxf(bm, l[j]);
    const float nm = fmaxf(mx, bm);
    if (nm == -INFINITY) continue;
    const float sc = mx == -INFINITY ? 0.f : expf(mx - nm);
    acc.x *= sc;
    acc.y *= sc;
    acc.z *= sc;
    acc.w *= sc;
    wsum *= sc;
#pragma unroll
    for (int j = 0; j < BLK; ++j) {
      const float w = l[j] == -INFINITY ? 0.f : expf(l[j] - nm);
      wsum += w;
      acc.x += w * v[j].x;
      acc.y += w * v[j].y;
      acc.z += w * v[j].z;
      acc.w += w * v[j].w;
    }
    mx = nm;
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  lse = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  o = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

}  // namespace tv
