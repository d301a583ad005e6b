// Tree-mask packing: keep-mask (int8 / bool, or additive float mask) ->
// one bit per (row, key).  The reference hands the Triton kernel an int8
// [B, M, M] mask converted on the host side of the call
// (tree_attention.py:449-460); the kernels here read 64 keys per 8-byte word.
#include "common.cuh"

namespace tv {
namespace {

__global__ void __launch_bounds__(256) pack_mask_kernel(int kind, const void* src, int64_t s_b, int64_t s_r,
                                                        int64_t s_c, int cols, uint64_t* out, int64_t out_sb,
                                                        int64_t out_sr) {
  const int b = blockIdx.z;
  const int r = blockIdx.y;
  const int c = blockIdx.x * 256 + threadIdx.x;
  bool keep = false;
  if (c < cols) {
    const int64_t off = (int64_t)b * s_b + (int64_t)r * s_r + (int64_t)c * s_c;
    switch (kind) {
      case 0: keep = static_cast<const int8_t*>(src)[off] != 0; break;
      case 1: keep = static_cast<const float*>(src)[off] == 0.f; break;
      case 2: keep = __half2float(static_cast<const __half*>(src)[off]) == 0.f; break;
      default: keep = __bfloat162float(static_cast<const __nv_bfloat16*>(src)[off]) == 0.f; break;
    }
  }
  const unsigned bits = __ballot_sync(0xffffffffu, keep);
  const int lane = threadIdx.x & 31;
  const int chunk = (blockIdx.x * 256 + (threadIdx.x & ~31)) >> 5;  // 32-bit chunk index within the row
  const int words = (cols + 63) >> 6;
  if (lane == 0 && chunk < 2 * words) {
    uint32_t* row = reinterpret_cast<uint32_t*>(out + (int64_t)b * out_sb + (int64_t)r * out_sr);
    row[chunk] = bits;  // little-endian: chunk 2w holds keys 64w..64w+31
  }
}

// 32 words per block; each word's rows are ANDed by 8 threads (rows g,
// g + 8, ...), whose results meet in shared memory: the loads of a column are
// in flight together instead of one after another.
__global__ void __launch_bounds__(256) mask_word_summary_kernel(const uint64_t* bits, int rows, int words, int64_t sb,
                                                                int64_t sr, uint8_t* out, int64_t out_sb) {
  __shared__ uint64_t part[8][32];
  const int b = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int g = threadIdx.x >> 5;
  const int w = blockIdx.x * 32 + lane;
  uint64_t acc = ~0ull;
  if (w < words) {
    const uint64_t* col = bits + (int64_t)b * sb + w;
    for (int r = g; r < rows; r += 8) acc &= col[(int64_t)r * sr];
  }
  part[g][lane] = acc;
  __syncthreads();
  if (g == 0 && w < words) {
#pragma unroll
    for (int k = 1; k < 8; ++k) acc &= part[k][lane];
    out[(int64_t)b * out_sb + w] = acc == ~0ull ? 1 : 0;
  }
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" int tv_mask_word_summary(const uint64_t* bits, int32_t batch, int32_t rows, int32_t words, int64_t sb,
                                    int64_t sr, uint8_t* out, int64_t out_sb, void* stream) {
  if (batch < 0 || rows < 0 || words < 0) return TV_ERR_SHAPE;
  if (batch == 0 || words == 0) return TV_OK;
  if (!bits || !out) return TV_ERR_NULL;
  if (sr < words || (batch > 1 && (sb < sr * rows || out_sb < words))) return TV_ERR_SHAPE;
  if (batch > 65535) return TV_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(bits) & 7) != 0) return TV_ERR_ALIGN;
  dim3 grid((words + 31) / 32, batch);
  mask_word_summary_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(bits, rows, words, sb, sr, out,
                                                                               out_sb);
  return check_launch();
}

extern "C" int tv_pack_mask(int32_t kind, const void* src, int64_t s_b, int64_t s_r, int64_t s_c, int32_t batch,
                            int32_t rows, int32_t cols, uint64_t* out, int64_t out_sb, int64_t out_sr, void* stream) {
  if (kind < 0 || kind > 3) return TV_ERR_DTYPE;
  if (batch < 0 || rows < 0 || cols < 0) return TV_ERR_SHAPE;
  if (batch == 0 || rows == 0 || cols == 0) return TV_OK;
  if (!src || !out) return TV_ERR_NULL;
  if (out_sr < (cols + 63) / 64 || (batch > 1 && out_sb < out_sr * rows)) return TV_ERR_SHAPE;
  if (rows > 65535 || batch > 65535) return TV_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(out) & 7) != 0) return TV_ERR_ALIGN;
  dim3 grid((cols + 255) / 256, rows, batch);
  pack_mask_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(kind, src, s_b, s_r, s_c, cols, out, out_sb,
                                                                        out_sr);
  return check_launch();
}
