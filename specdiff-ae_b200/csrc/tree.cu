// Final draft-tree build on the device: DraftTree.update's final branch and
// generate_attention_mask (runtime/draft_tree.py:188-260) plus the root row /
// column of the verify mask (diffspec_model.py:620-624), in one CTA and one
// launch.  The reference walks the ancestors with a host sync per hop.
//
// Thread t takes top-k entry t: its depth row and column, its final position
// (entries ordered by depth, top-k order kept among equal depths), the
// position table, then its parent position and its row of the masks.
#include "common.cuh"
#include "specverify.h"

namespace tv {
namespace {

constexpr int kMaxK = 1024;
constexpr int kMaxTable = 8192;    // depth * nnodes entries of the position table

__global__ void __launch_bounds__(kMaxK) tree_finalize_kernel(int nnodes, int depth, int k, const int64_t* top,
                                                              const int64_t* pm, int64_t pm_s, const int64_t* im,
                                                              int64_t im_s, const int64_t* d2t, int64_t d2t_len,
                                                              int64_t* ids_out, int64_t* pos_out, int64_t* par_out,
                                                              int8_t* mask, uint64_t* bits, int* status) {
  __shared__ int s_row[kMaxK];        // depth row of top-k entry t
  __shared__ int s_par[kMaxK];        // parent position of final position p
  __shared__ int table[kMaxTable];    // [depth][nnodes] -> final position
  __shared__ int bad;
  const int t = threadIdx.x;
  if (t == 0) bad = 0;
  for (int i = t; i < depth * nnodes; i += blockDim.x) table[i] = -1;
  int r = 0, c = 0;
  if (t < k) {
    const int64_t key = top[t];
    if (key < 0 || key >= (int64_t)depth * nnodes) {
      bad = 1;
    } else {
      r = (int)(key / nnodes);
      c = (int)(key - (int64_t)r * nnodes);
    }
    s_row[t] = r;
  }
  __syncthreads();
  int p = 0;
  if (t < k) {
    // final position: entries of smaller depth, then earlier entries of the same depth
    for (int j = 0; j < k; ++j) p += (s_row[j] < r) || (s_row[j] == r && j < t);
    if (atomicExch(&table[r * nnodes + c], p) != -1) bad = 1;   // repeated index
  }
  __syncthreads();
  if (t < k) {
    const int64_t pc = pm[(int64_t)r * pm_s + c];
    int pp = -1;
    if (r > 0 && pc >= 0 && pc < nnodes) pp = table[(r - 1) * nnodes + (int)pc];
    s_par[p] = pp;
    int64_t id = im[(int64_t)r * im_s + c];
    if (d2t) {
      if (id < 0 || id >= d2t_len) bad = 1;
      else id += d2t[id];
    }
    ids_out[p] = id;
    pos_out[p] = r + 1;
    par_out[p] = pp;
  }
  __syncthreads();
  if (t < k) {
    // thread t now takes final position t: its mask row holds itself and its
    // ancestors (at most depth - 1 hops)
    if (mask) {
      int8_t* row = mask + (int64_t)t * k;
      for (int j = 0; j < k; ++j) row[j] = j == t;
    }
    const int words = (k + 1 + 63) / 64;
    uint64_t* brow = bits ? bits + (int64_t)(t + 1) * words : nullptr;
    if (brow) {
      for (int w = 0; w < words; ++w) brow[w] = 0;
    }
    int cur = s_par[t];
    for (int h = 0; h < depth - 1 && cur >= 0 && cur < k; ++h) {
      if (mask) mask[(int64_t)t * k + cur] = 1;
      if (brow) brow[(cur + 1) >> 6] |= 1ull << ((cur + 1) & 63);
      cur = s_par[cur];
    }
    if (brow) {
      brow[0] |= 1ull;                                   // the root column
      brow[(t + 1) >> 6] |= 1ull << ((t + 1) & 63);      // itself
    }
    if (t == 0 && bits) {                                // the root row sees only itself
      bits[0] = 1ull;
      for (int w = 1; w < words; ++w) bits[w] = 0;
    }
  }
  __syncthreads();
  if (t == 0 && bad && status) atomicExch(status, TV_ERR_INPUT);
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" int tv_tree_finalize(int32_t nnodes, int32_t depth, int32_t k, const int64_t* top_index,
                                const int64_t* parents_matrix, int64_t pm_stride, const int64_t* input_ids_matrix,
                                int64_t im_stride, const int64_t* d2t, int64_t d2t_len, int64_t* input_ids,
                                int64_t* position_ids, int64_t* parent_pos, int8_t* mask, uint64_t* mask_bits,
                                int32_t* status, void* stream) {
  if (nnodes < 1 || depth < 1 || k < 0) return TV_ERR_SHAPE;
  if (k > kMaxK || (int64_t)depth * nnodes > kMaxTable) return TV_ERR_UNSUPPORTED;
  if (k == 0) return TV_OK;
  if (!top_index || !parents_matrix || !input_ids_matrix || !input_ids || !position_ids || !parent_pos)
    return TV_ERR_NULL;
  if (pm_stride < nnodes || im_stride < nnodes) return TV_ERR_SHAPE;
  if (d2t && d2t_len < 1) return TV_ERR_SHAPE;
  if (mask_bits && (reinterpret_cast<uintptr_t>(mask_bits) & 7) != 0) return TV_ERR_ALIGN;
  const int threads = ((k + 31) / 32) * 32;
  tree_finalize_kernel<<<1, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      nnodes, depth, k, top_index, parents_matrix, pm_stride, input_ids_matrix, im_stride, d2t, d2t_len, input_ids,
      position_ids, parent_pos, mask, mask_bits, status);
  return check_launch();
}
