// Host-side launchers of the verify-attention kernels.
#pragma once

#include <cuda_runtime.h>

#include "attn_params.cuh"

namespace tv {

// Warp-MMA (mma.sync) path: any row count, head_dim 32, 64 or 128.
// precise: softmax weights enter PV as a hi + lo 16-bit pair.
int launch_attn_mma(const AttnParams& p, int dtype, int D, bool precise, cudaStream_t st);
int mma_tile_keys();
int mma_row_blocks(int R);   // CTAs per (batch, KV head)

// Tensor-memory (tcgen05) path: head_dim 128, >= 64 query rows per KV head.
// kernel_bits: tv_attn_args.kernel (bit 7 forces half-head TMA boxes).
int launch_attn_tc(const AttnParams& p, int dtype, int D, int kernel_bits, cudaStream_t st);
// 1 when launch_attn_tc would load whole-head (wide) TMA boxes for p.
int attn_tc_wide(const AttnParams& p, int dtype, int kernel_bits);
bool tc_supported(int dtype, int D, int R, bool paged, int page_shift);
int tc_tile_keys();
int tc_rows_per_cta();
int tc_row_blocks(int R);   // CTAs per (batch, KV head)

// Log-sum-exp merge of split partials into the final outputs of AttnParams.
int launch_split_combine(const AttnParams& p, int dtype, int D, cudaStream_t st);

// Sequence-sharded step, after the attention kernel left this rank's split
// partials in p.part_o / p.part_lse: combine them, exchange them with the
// peers over NVLink (pushed to every peer, or -- `owned` -- to the rank that
// owns each row block, which merges and hands the final rows back) and write
// the merged final outputs of AttnParams (same on every rank).
constexpr int kMaxPeers = 8;
int launch_sharded_combine(const AttnParams& p, int dtype, int D, int world, int rank, const void* const* bases,
                           bool owned, cudaStream_t st);
// Bytes of one rank's exchange buffer (the layout launch_sharded_combine uses).
int64_t sharded_exchange_bytes(int world, int64_t rows, int D);

}  // namespace tv
