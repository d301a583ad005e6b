// Accepted-path KV compaction and working-set staging, as coalesced
// 128-bit copies (narrower only when a caller's alignment forces it).
//
//   tv_compact_contig     contiguous cache, diffspec/draft/tree_verification.py:197-217
//   tv_copy_pages         copy-on-write page copies, diffspec/core/kv_cache/paged_kv.py:208-220
//   tv_compact_paged      path compaction through a page table
//   tv_arena_gather       chunk arena staging, diffspec/core/kv_cache/chunk_arena.py:126-173
//   tv_gather_page_table  zero-copy arena: the working set as a page-table view
//
// Row moves read every source row of a slice into shared memory before any
// write, the gather-then-write order of the reference's
// `data[..., idx, :]` followed by `dst.copy_(tgt)`.
#include "common.cuh"

namespace tv {
namespace {

constexpr int CT = 128;

// Widest copy unit (bytes) that every address and stride allows.
int unit_for(uintptr_t bits) {
  if ((bits & 15) == 0) return 16;
  if ((bits & 7) == 0) return 8;
  if ((bits & 3) == 0) return 4;
  if ((bits & 1) == 0) return 2;
  return 1;
}

template <typename U>
__device__ __forceinline__ void copy_row_to_smem(uint8_t* dst, const uint8_t* src, int row_bytes, int tid) {
  for (int o = tid * (int)sizeof(U); o < row_bytes; o += CT * (int)sizeof(U))
    *reinterpret_cast<U*>(dst + o) = src ? *reinterpret_cast<const U*>(src + o) : U{};
}
template <typename U>
__device__ __forceinline__ void copy_row_from_smem(uint8_t* dst, const uint8_t* src, int row_bytes, int tid) {
  for (int o = tid * (int)sizeof(U); o < row_bytes; o += CT * (int)sizeof(U))
    *reinterpret_cast<U*>(dst + o) = *reinterpret_cast<const U*>(src + o);
}

template <typename U>
__global__ void __launch_bounds__(CT) compact_contig_kernel(uint8_t* data, int64_t num_slices, int64_t slice_stride,
                                                            int64_t row_stride, int row_bytes, int64_t start,
                                                            const int64_t* res, int max_rows) {
  extern __shared__ __align__(16) uint8_t buf[];
  if (res[0] != 0) return;
  const int n = (int)(res[2] < (int64_t)max_rows ? res[2] : (int64_t)max_rows);
  const int64_t* path = res + 8;
  for (int64_t s = blockIdx.x; s < num_slices; s += gridDim.x) {
    uint8_t* base = data + s * slice_stride;
    for (int j = 0; j < n; ++j)
      copy_row_to_smem<U>(buf + (size_t)j * row_bytes, base + (start + path[j]) * row_stride, row_bytes, threadIdx.x);
    __syncthreads();
    for (int j = 0; j < n; ++j)
      copy_row_from_smem<U>(base + (start + j) * row_stride, buf + (size_t)j * row_bytes, row_bytes, threadIdx.x);
    __syncthreads();
  }
}

template <typename U>
__global__ void __launch_bounds__(256) copy_pages_kernel(uint8_t* pool, int64_t plane_stride, int64_t page_stride,
                                                         int64_t page_bytes, const int32_t* pairs, int num_pages) {
  const int pr = blockIdx.x;
  const int plane = blockIdx.y;
  const int src = pairs[2 * pr], dst = pairs[2 * pr + 1];
  if (src < 0 || src >= num_pages || dst < 0 || dst >= num_pages || src == dst) return;
  const uint8_t* s = pool + plane * plane_stride + (int64_t)src * page_stride;
  uint8_t* d = pool + plane * plane_stride + (int64_t)dst * page_stride;
  for (int64_t o = (int64_t)threadIdx.x * sizeof(U); o < page_bytes; o += 256 * (int64_t)sizeof(U))
    *reinterpret_cast<U*>(d + o) = *reinterpret_cast<const U*>(s + o);
}

template <typename U>
__global__ void __launch_bounds__(CT) compact_paged_kernel(uint8_t* pool, int64_t plane_stride, int64_t page_stride,
                                                           int64_t head_stride, int64_t row_stride, int row_bytes,
                                                           int page_shift, const int32_t* src_table,
                                                           const int32_t* dst_table, int table_len,
                                                           int num_pages, int64_t start, const int64_t* res,
                                                           int max_rows) {
  extern __shared__ __align__(16) uint8_t buf[];
  if (res[0] != 0) return;
  const int n = (int)(res[2] < (int64_t)max_rows ? res[2] : (int64_t)max_rows);
  const int64_t* path = res + 8;
  const int plane = blockIdx.x, head = blockIdx.y;
  uint8_t* base = pool + plane * plane_stride + head * head_stride;
  const int64_t pmask = (1LL << page_shift) - 1;
  for (int j = 0; j < n; ++j) {
    const int64_t tok = start + path[j];
    const int64_t lp = tok >> page_shift;
    const int page = (lp >= 0 && lp < table_len) ? src_table[lp] : -1;
    const uint8_t* src = (page >= 0 && page < num_pages) ? base + (int64_t)page * page_stride + (tok & pmask) * row_stride
                                                         : nullptr;
    copy_row_to_smem<U>(buf + (size_t)j * row_bytes, src, row_bytes, threadIdx.x);
  }
  __syncthreads();
  for (int j = 0; j < n; ++j) {
    const int64_t tok = start + j;
    const int64_t lp = tok >> page_shift;
    const int page = (lp >= 0 && lp < table_len) ? dst_table[lp] : -1;
    if (page < 0 || page >= num_pages) continue;
    copy_row_from_smem<U>(base + (int64_t)page * page_stride + (tok & pmask) * row_stride, buf + (size_t)j * row_bytes,
                          row_bytes, threadIdx.x);
  }
}

template <typename U>
__global__ void __launch_bounds__(CT) arena_gather_kernel(int heads, const uint64_t* src_k, const uint64_t* src_v,
                                                          int64_t src_head_stride, int64_t src_row_stride,
                                                          int src_len, uint8_t* arena, int64_t layer_stride,
                                                          int64_t kv_stride, int64_t head_stride, int row_bytes,
                                                          int chunk, int arena_rows, const int32_t* copies) {
  const int cp = blockIdx.x;
  const int layer = blockIdx.y >> 1, kv = blockIdx.y & 1;
  const int head = blockIdx.z;
  const int c = copies[2 * cp], slot = copies[2 * cp + 1];
  const int64_t r0 = (int64_t)c * chunk;
  const int64_t r1 = (r0 + chunk < (int64_t)src_len ? r0 + chunk : (int64_t)src_len);
  if (c < 0 || slot < 0 || (int64_t)(slot + 1) * chunk > arena_rows) return;
  const uint8_t* s = reinterpret_cast<const uint8_t*>(kv ? src_v[layer] : src_k[layer]) + head * src_head_stride;
  uint8_t* d = arena + layer * layer_stride + kv * kv_stride + head * head_stride + (int64_t)slot * chunk * row_bytes;
  const int per_row = row_bytes / (int)sizeof(U);
  const int64_t rows = r1 - r0;
  if (per_row <= CT && CT % per_row == 0) {
    // A thread keeps one column of the row and walks the rows CT / per_row
    // apart, four loads in flight before their stores (no 64-bit divisions).
    const int64_t col = (int64_t)(threadIdx.x % per_row) * sizeof(U);
    const int rstep = CT / per_row;
    const uint8_t* sc = s + r0 * src_row_stride + col;
    uint8_t* dc = d + col;
    int64_t r = threadIdx.x / per_row;
    for (; r + 3 * rstep < rows; r += 4 * rstep) {
      U v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) v[k] = *reinterpret_cast<const U*>(sc + (r + k * rstep) * src_row_stride);
#pragma unroll
      for (int k = 0; k < 4; ++k) *reinterpret_cast<U*>(dc + (r + k * rstep) * row_bytes) = v[k];
    }
    for (; r < rows; r += rstep)
      *reinterpret_cast<U*>(dc + r * row_bytes) = *reinterpret_cast<const U*>(sc + r * src_row_stride);
    return;
  }
  const int64_t total = rows * per_row;
  for (int64_t e = threadIdx.x; e < total; e += CT) {
    const int64_t r = e / per_row;
    const int64_t o = (e - r * per_row) * sizeof(U);
    *reinterpret_cast<U*>(d + r * row_bytes + o) = *reinterpret_cast<const U*>(s + (r0 + r) * src_row_stride + o);
  }
}

__global__ void gather_table_kernel(const int32_t* table, int table_len, const int32_t* ids, int nchunks, int ppc,
                                    int32_t* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nchunks * ppc) return;
  const int64_t lp = (int64_t)ids[i / ppc] * ppc + (i % ppc);
  out[i] = (lp >= 0 && lp < table_len) ? table[lp] : -1;
}

// Calls f(U{}) with U the copy unit of `u` bytes.
template <typename F>
void dispatch_unit(int u, F&& f) {
  switch (u) {
    case 16: f(uint4{}); break;
    case 8: f(uint2{}); break;
    case 4: f(uint32_t{}); break;
    case 2: f(uint16_t{}); break;
    default: f(uint8_t{}); break;
  }
}

int set_smem(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return TV_OK;
  if (bytes > 227 * 1024) return TV_ERR_UNSUPPORTED;
  return ensure_dynamic_smem(reinterpret_cast<const void*>(fn), (int)bytes);
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" {

int tv_compact_contig(void* data, int64_t num_slices, int64_t slice_stride_bytes, int64_t row_stride_bytes,
                      int32_t row_bytes, int64_t start, const int64_t* accept_result, int32_t max_rows, void* stream) {
  if (num_slices < 0 || row_bytes <= 0 || max_rows <= 0 || start < 0) return TV_ERR_SHAPE;
  if (num_slices == 0) return TV_OK;
  if (!data || !accept_result) return TV_ERR_NULL;
  const int u = unit_for(reinterpret_cast<uintptr_t>(data) | (uintptr_t)slice_stride_bytes |
                         (uintptr_t)row_stride_bytes | (uintptr_t)row_bytes);
  const size_t smem = (size_t)max_rows * row_bytes;
  const unsigned grid = (unsigned)(num_slices < 65535 ? num_slices : 65535);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = TV_OK;
  dispatch_unit(u, [&](auto tag) {
    using U = decltype(tag);
    rc = set_smem((const void*)compact_contig_kernel<U>, smem);
    if (rc == TV_OK)
      compact_contig_kernel<U><<<grid, CT, smem, st>>>(static_cast<uint8_t*>(data), num_slices, slice_stride_bytes,
                                                       row_stride_bytes, row_bytes, start, accept_result, max_rows);
  });
  if (rc != TV_OK) return rc;
  return check_launch();
}

int tv_copy_pages(void* pool, int32_t planes, int64_t plane_stride_bytes, int64_t page_stride_bytes,
                  int64_t page_bytes, const int32_t* pairs, int32_t npairs, int32_t num_pages, void* stream) {
  if (planes < 0 || npairs < 0 || page_bytes <= 0 || num_pages <= 0) return TV_ERR_SHAPE;
  if (planes == 0 || npairs == 0) return TV_OK;
  if (!pool || !pairs) return TV_ERR_NULL;
  if (planes > 65535 || npairs > 0x7fffffff) return TV_ERR_SHAPE;
  const int u = unit_for(reinterpret_cast<uintptr_t>(pool) | (uintptr_t)plane_stride_bytes |
                         (uintptr_t)page_stride_bytes | (uintptr_t)page_bytes);
  dim3 grid(npairs, planes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dispatch_unit(u, [&](auto tag) {
    using U = decltype(tag);
    copy_pages_kernel<U><<<grid, 256, 0, st>>>(static_cast<uint8_t*>(pool), plane_stride_bytes, page_stride_bytes,
                                               page_bytes, pairs, num_pages);
  });
  return check_launch();
}

int tv_compact_paged(void* pool, int32_t planes, int32_t heads, int64_t plane_stride_bytes, int64_t page_stride_bytes,
                     int64_t head_stride_bytes, int64_t row_stride_bytes, int32_t row_bytes, int32_t page_size,
                     const int32_t* src_table, const int32_t* dst_table, int32_t table_len, int32_t num_pages,
                     int64_t start, const int64_t* accept_result, int32_t max_rows, void* stream) {
  if (planes < 0 || heads < 0 || row_bytes <= 0 || max_rows <= 0 || start < 0 || num_pages <= 0) return TV_ERR_SHAPE;
  if (page_size <= 0 || (page_size & (page_size - 1))) return TV_ERR_UNSUPPORTED;
  if (planes == 0 || heads == 0) return TV_OK;
  if (!pool || !src_table || !dst_table || !accept_result) return TV_ERR_NULL;
  if (planes > 0x7fffffff || heads > 65535) return TV_ERR_SHAPE;
  int shift = 0;
  while ((1 << shift) < page_size) ++shift;
  const int u = unit_for(reinterpret_cast<uintptr_t>(pool) | (uintptr_t)plane_stride_bytes |
                         (uintptr_t)page_stride_bytes | (uintptr_t)head_stride_bytes | (uintptr_t)row_stride_bytes |
                         (uintptr_t)row_bytes);
  const size_t smem = (size_t)max_rows * row_bytes;
  dim3 grid(planes, heads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = TV_OK;
  dispatch_unit(u, [&](auto tag) {
    using U = decltype(tag);
    rc = set_smem((const void*)compact_paged_kernel<U>, smem);
    if (rc == TV_OK)
      compact_paged_kernel<U><<<grid, CT, smem, st>>>(static_cast<uint8_t*>(pool), plane_stride_bytes,
                                                      page_stride_bytes, head_stride_bytes, row_stride_bytes,
                                                      row_bytes, shift, src_table, dst_table, table_len, num_pages, start,
                                                      accept_result, max_rows);
  });
  if (rc != TV_OK) return rc;
  return check_launch();
}

int tv_arena_gather(int32_t layers, int32_t heads, const uint64_t* src_k, const uint64_t* src_v,
                    int64_t src_head_stride_bytes, int64_t src_row_stride_bytes, int32_t src_len, void* arena,
                    int64_t arena_layer_stride_bytes, int64_t arena_kv_stride_bytes, int64_t arena_head_stride_bytes,
                    int32_t row_bytes, int32_t chunk_size, int32_t arena_rows, const int32_t* copies, int32_t ncopies,
                    void* stream) {
  if (layers < 0 || heads < 0 || row_bytes <= 0 || chunk_size <= 0 || ncopies < 0 || src_len < 0) return TV_ERR_SHAPE;
  if (layers == 0 || heads == 0 || ncopies == 0) return TV_OK;
  if (!src_k || !src_v || !arena || !copies) return TV_ERR_NULL;
  if (2 * layers > 65535 || heads > 65535) return TV_ERR_SHAPE;
  const int u = unit_for(reinterpret_cast<uintptr_t>(arena) | (uintptr_t)src_head_stride_bytes |
                         (uintptr_t)src_row_stride_bytes | (uintptr_t)arena_layer_stride_bytes |
                         (uintptr_t)arena_kv_stride_bytes | (uintptr_t)arena_head_stride_bytes | (uintptr_t)row_bytes);
  dim3 grid(ncopies, 2 * layers, heads);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dispatch_unit(u, [&](auto tag) {
    using U = decltype(tag);
    arena_gather_kernel<U><<<grid, CT, 0, st>>>(heads, src_k, src_v, src_head_stride_bytes, src_row_stride_bytes,
                                                src_len, static_cast<uint8_t*>(arena), arena_layer_stride_bytes,
                                                arena_kv_stride_bytes, arena_head_stride_bytes, row_bytes,
                                                chunk_size, arena_rows, copies);
  });
  return check_launch();
}

int tv_gather_page_table(const int32_t* page_table, int32_t table_len, const int32_t* chunk_ids, int32_t nchunks,
                         int32_t pages_per_chunk, int32_t* out, void* stream) {
  if (nchunks < 0 || pages_per_chunk <= 0 || table_len < 0) return TV_ERR_SHAPE;
  if (nchunks == 0) return TV_OK;
  if (!page_table || !chunk_ids || !out) return TV_ERR_NULL;
  const int n = nchunks * pages_per_chunk;
  gather_table_kernel<<<(n + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(page_table, table_len, chunk_ids,
                                                                                       nchunks, pages_per_chunk, out);
  return check_launch();
}

}  // extern "C"
