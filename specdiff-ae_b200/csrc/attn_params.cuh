// Launch parameters shared by the verify-attention kernels.
#pragma once

#include <stdint.h>

namespace tv {

struct AttnParams {
  const void* q;
  int64_t q_sb, q_sm, q_sh;
  const void* k;
  const void* v;
  int64_t k_sb, k_sn, k_sh;
  int64_t v_sb, v_sn, v_sh;
  const int32_t* pt;      // page table (nullptr = contiguous)
  int64_t pt_sb;
  int page_shift;         // log2(page_size)
  int num_pages;
  const int32_t* kv_lens;
  int num_keys;
  int mask_len;
  const uint64_t* mask;
  int64_t mask_sb, mask_sm;
  const uint8_t* mfull;    // optional per (batch, mask word): all rows see all 64 keys
  int64_t mfull_sb;
  int B, M, H, Hkv, G, R;  // R = M * G query rows per (batch, kv head)
  float scale_log2;        // softmax scale * log2(e)
  int splits;
  int tiles_per_split;     // key tiles (of the kernel's tile size) per split
  // final outputs
  void* out;
  int64_t o_sb, o_sm, o_sh;
  int out_f32;
  float* lse;
  int64_t lse_sb, lse_sm, lse_sh;
  const float* aux;
  int64_t aux_sb, aux_sm, aux_sh;
  void* weight;
  int64_t w_sb, w_sm, w_sh;
  // split partials: [splits][B*Hkv][R][D] and [splits][B*Hkv][R].  When set
  // (always with splits > 1; also with one split for the sharded path), the
  // kernels write normalised partials here instead of the final outputs.
  float* part_o;
  float* part_lse;
  int* err;                // optional device status word (nonzero = a wait gave up)
};

}  // namespace tv
