// Draft-side chunk retrieval (sm_100a): the retrieval branch of
// DraftNetwork._select_working_cache_from_chunks (draft_network.py:1514-1612)
// -- chunk scores from the per-token attention, top-k chunks, the union of
// their token intervals, and the gather of those token rows of every layer's
// K and V -- without the host round trips of the reference (.any(),
// .tolist(), nonzero).
//
// tv_chunk_select: a grid kernel sums every chunk's attention in double
// (one CTA per chunk) and finds where the scores first turn NaN / +-inf;
// then one CTA rounds the sums to float (the reference subtracts float
// prefix sums; for exactly representable scores the two agree bit for bit),
// ranks the chunks in the torch.topk order (NaN first, then larger, then
// smaller id), orders the selected intervals by start and merges them; a
// grid kernel expands the merged runs into ascending token indices.
// tv_gather_rows: a copy in 16-byte units, one grid row per (plane, head),
// four units per thread with the loads ahead of the stores; the row count is
// read on the device.
#include "accept_common.cuh"

namespace tv {
namespace {

constexpr int SEL_THREADS = 1024;
constexpr int kMaxChunks = 2048;
constexpr int kMaxTopK = 1024;
constexpr int SCAN_BLOCK = 8192;          // attention scores per block of the non-finite scan

__device__ __forceinline__ void chunk_bounds(const int64_t* starts, const int64_t* ends, int c, int64_t la,
                                             int64_t& lo, int64_t& hi) {
  const int64_t s = starts[c], e = ends[c];
  lo = s > 0 ? min(max(s - 1, (int64_t)0), la - 1) + 1 : 0;   // prefix length below the chunk
  hi = min(max(e - 1, (int64_t)0), la - 1) + 1;
}

// Blocks [0, n): chunk c's attention sum over [min(lo, hi), max(lo, hi)) in
// double.  Blocks [n, n + scan blocks): the first NaN / +inf / -inf of one
// slice of the scores (la where there is none).
__global__ void __launch_bounds__(256) chunk_sums_kernel(const float* attn, int64_t la, const int64_t* starts,
                                                         const int64_t* ends, int n, double* sums,
                                                         long long* firsts) {
  __shared__ double red[8];
  __shared__ unsigned long long f[3];
  const int tid = threadIdx.x;
  if ((int)blockIdx.x < n) {
    int64_t lo, hi;
    chunk_bounds(starts, ends, blockIdx.x, la, lo, hi);
    const int64_t a = min(lo, hi), b = max(lo, hi);
    double acc[4] = {0.0, 0.0, 0.0, 0.0};
    for (int64_t t0 = a + tid; t0 < b; t0 += 256 * 8) {
      float x[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t t = t0 + 256 * u;
        x[u] = t < b ? __ldg(attn + t) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u & 3] += (double)x[u];
    }
    double v = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((tid & 31) == 0) red[tid >> 5] = v;
    __syncthreads();
    if (tid == 0) {
      double t = 0.0;
      for (int w = 0; w < 8; ++w) t += red[w];
      sums[blockIdx.x] = t;
    }
    return;
  }
  const int64_t base = (int64_t)(blockIdx.x - n) * SCAN_BLOCK;
  if (tid < 3) f[tid] = (unsigned long long)la;
  __syncthreads();
  float x[SCAN_BLOCK / 256];
#pragma unroll
  for (int u = 0; u < SCAN_BLOCK / 256; ++u) {
    const int64_t t = base + tid + 256 * u;
    x[u] = t < la ? __ldg(attn + t) : 0.f;
  }
#pragma unroll
  for (int u = 0; u < SCAN_BLOCK / 256; ++u) {
    const int64_t t = base + tid + 256 * u;
    if (x[u] != x[u]) atomicMin(&f[0], (unsigned long long)t);
    else if (x[u] == INFINITY) atomicMin(&f[1], (unsigned long long)t);
    else if (x[u] == -INFINITY) atomicMin(&f[2], (unsigned long long)t);
  }
  __syncthreads();
  if (tid < 3) firsts[(int64_t)(blockIdx.x - n) * 3 + tid] = (long long)f[tid];
}

__global__ void __launch_bounds__(SEL_THREADS) chunk_select_kernel(int64_t la, const int64_t* starts,
                                                                   const int64_t* ends, int n, int k, int64_t length,
                                                                   const double* sums, const long long* firsts,
                                                                   int nscan, int64_t* selected, int64_t* run_start,
                                                                   int64_t* run_off, int* run_count,
                                                                   int64_t max_indices, int64_t* count, int* status) {
  __shared__ float s_score[kMaxChunks];
  __shared__ int s_pos[kMaxChunks];        // position among the selected (ascending id), or -1
  __shared__ int64_t s_a[kMaxTopK];        // selected intervals, then merged runs
  __shared__ int64_t s_b[kMaxTopK];
  __shared__ int64_t s_off[kMaxTopK + 1];
  __shared__ int s_runs, s_bad;
  __shared__ unsigned long long s_first[3];   // first NaN, +inf, -inf in attn (la if none)
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_bad = 0;
    s_first[0] = s_first[1] = s_first[2] = (unsigned long long)la;
  }
  __syncthreads();
  for (int i = tid; i < 3 * nscan; i += SEL_THREADS) atomicMin(&s_first[i % 3], (unsigned long long)firsts[i]);
  __syncthreads();
  // where the reference's float prefix sums turn non-finite: a chunk's score
  // then follows IEEE arithmetic on those prefix sums (a NaN makes every later
  // prefix, and so every chunk ending after it, NaN)
  const int64_t f_nan = (int64_t)s_first[0], f_pinf = (int64_t)s_first[1], f_ninf = (int64_t)s_first[2];
  auto prefix_special = [&](int64_t x, bool& finite) -> float {
    finite = false;
    if (f_nan < x || (f_pinf < x && f_ninf < x)) return __int_as_float(0x7fc00000);
    if (f_pinf < x) return INFINITY;
    if (f_ninf < x) return -INFINITY;
    finite = true;
    return 0.f;
  };
  // 1. chunk scores
  for (int c = tid; c < n; c += SEL_THREADS) {
    const int64_t s = starts[c], e = ends[c];
    if (s < 0 || e < 0) s_bad = 1;
    int64_t lo, hi;
    chunk_bounds(starts, ends, c, la, lo, hi);
    bool fin_hi, fin_lo;
    const float sp_hi = prefix_special(hi, fin_hi), sp_lo = prefix_special(lo, fin_lo);
    const float fs = (fin_hi && fin_lo) ? (float)(hi >= lo ? sums[c] : -sums[c]) : sp_hi - sp_lo;
    const float len = (float)(e - s > 1 ? e - s : 1);
    s_score[c] = fs / len;
  }
  __syncthreads();
  // 2. top-k by rank: the chunks that fewer than k others beat
  for (int c = tid; c < n; c += SEL_THREADS) {
    int rank = 0;
    for (int j = 0; j < n; ++j) rank += acc::better(s_score[j], j, s_score[c], c);
    s_pos[c] = rank < k ? 1 : 0;
  }
  __syncthreads();
  // 3. ascending ids of the selected chunks (serial prefix over at most 2048 flags)
  if (tid == 0) {
    int p = 0;
    for (int c = 0; c < n; ++c) s_pos[c] = s_pos[c] ? p++ : -1;
  }
  __syncthreads();
  for (int c = tid; c < n; c += SEL_THREADS) {
    const int p = s_pos[c];
    if (p >= 0) {
      selected[p] = c;
      s_a[p] = min(max(starts[c], (int64_t)0), length);
      s_b[p] = min(max(ends[c], (int64_t)0), length);
    }
  }
  __syncthreads();
  // 4. order the intervals by start and merge overlapping / touching ones
  if (tid == 0) {
    // insertion sort by (start, end): k <= 1024 intervals, nearly sorted already
    for (int i = 1; i < k; ++i) {
      const int64_t a = s_a[i], b = s_b[i];
      int j = i - 1;
      while (j >= 0 && (s_a[j] > a || (s_a[j] == a && s_b[j] > b))) {
        s_a[j + 1] = s_a[j];
        s_b[j + 1] = s_b[j];
        --j;
      }
      s_a[j + 1] = a;
      s_b[j + 1] = b;
    }
    int r = 0;
    for (int i = 0; i < k; ++i) {
      if (s_b[i] <= s_a[i]) continue;                       // empty interval
      if (r > 0 && s_a[i] <= s_b[r - 1]) {
        if (s_b[i] > s_b[r - 1]) s_b[r - 1] = s_b[i];
      } else {
        s_a[r] = s_a[i];
        s_b[r] = s_b[i];
        ++r;
      }
    }
    s_off[0] = 0;
    for (int i = 0; i < r; ++i) s_off[i + 1] = s_off[i] + (s_b[i] - s_a[i]);
    s_runs = r;
    int64_t total = s_off[r];
    if (total > max_indices) {
      s_bad = 1;
      total = max_indices;
    }
    *count = total;
    *run_count = r;
  }
  __syncthreads();
  // 5. the merged runs, for the expansion into token indices
  for (int i = tid; i <= s_runs; i += SEL_THREADS) {
    run_off[i] = s_off[i];
    if (i < s_runs) run_start[i] = s_a[i];
  }
  if (tid == 0 && s_bad && status) atomicExch(status, TV_ERR_INPUT);
}

// Token t of the union (t < count): run r with run_off[r] <= t < run_off[r + 1]
// (binary search), index run_start[r] + t - run_off[r].
__global__ void __launch_bounds__(256) expand_runs_kernel(const int64_t* run_start, const int64_t* run_off,
                                                          const int* run_count, const int64_t* count,
                                                          int64_t* indices) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= *count) return;
  int lo = 0, hi = *run_count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (run_off[mid] <= t) lo = mid;
    else hi = mid - 1;
  }
  indices[t] = run_start[lo] + (t - run_off[lo]);
}

// blockIdx.y = plane * heads + head; thread units of 16 bytes along the
// output rows, four per thread with every load issued before the stores.
__global__ void __launch_bounds__(256) gather_rows_kernel(int heads, const uint64_t* src, const uint64_t* dst,
                                                          int64_t shs, int64_t srs, int64_t dhs, int64_t drs,
                                                          int upr, const int64_t* indices, const int64_t* count,
                                                          int64_t max_rows) {
  const int n = (int)min(*count, max_rows);
  const int units = n * upr;
  const int p = blockIdx.y / heads, h = blockIdx.y - p * heads;
  const uint8_t* sbase = reinterpret_cast<const uint8_t*>(src[p]) + h * shs;
  uint8_t* dbase = reinterpret_cast<uint8_t*>(dst[p]) + h * dhs;
  const int stride = gridDim.x * blockDim.x;
  for (int u0 = blockIdx.x * blockDim.x + threadIdx.x; u0 < units; u0 += 4 * stride) {
    uint4 v[4];
    int64_t doff[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int u = u0 + k * stride;
      doff[k] = -1;
      if (u < units) {
        const int i = u / upr, part = u - i * upr;
        v[k] = __ldg(reinterpret_cast<const uint4*>(sbase + __ldg(indices + i) * srs) + part);
        doff[k] = i * drs + part * 16;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (doff[k] >= 0) *reinterpret_cast<uint4*>(dbase + doff[k]) = v[k];
  }
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" {

int tv_chunk_select_workspace_size(int32_t nchunks, int64_t attn_len, size_t* bytes) {
  if (!bytes) return TV_ERR_NULL;
  if (nchunks < 0 || attn_len < 0) return TV_ERR_SHAPE;
  const int64_t nscan = (attn_len + SCAN_BLOCK - 1) / SCAN_BLOCK;
  // chunk sums, per-slice first non-finite scores, merged runs (start, offset), run count
  *bytes = (size_t)nchunks * sizeof(double) + (size_t)nscan * 3 * sizeof(long long) +
           (size_t)(2 * kMaxTopK + 1) * sizeof(int64_t) + 64;
  return TV_OK;
}

int tv_chunk_select(const float* attn, int64_t attn_len, const int64_t* starts, const int64_t* ends,
                    int32_t nchunks, int32_t top_k, int64_t length, int64_t* selected, int64_t* indices,
                    int64_t max_indices, int64_t* count, void* workspace, size_t workspace_bytes,
                    int32_t* status, void* stream) {
  if (nchunks < 0 || top_k < 0 || length < 0 || max_indices < 0) return TV_ERR_SHAPE;
  if (nchunks > kMaxChunks) return TV_ERR_UNSUPPORTED;
  if (!count) return TV_ERR_NULL;
  const int k = top_k < nchunks ? top_k : nchunks;
  if (k > kMaxTopK) return TV_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k == 0) {
    const cudaError_t e = cudaMemsetAsync(count, 0, sizeof(int64_t), st);
    return e == cudaSuccess ? TV_OK : record_cuda_error(e);
  }
  if (!attn || attn_len < 1 || !starts || !ends || !selected || !indices) return TV_ERR_NULL;
  size_t need = 0;
  tv_chunk_select_workspace_size(nchunks, attn_len, &need);
  if (!workspace || workspace_bytes < need) return TV_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return TV_ERR_ALIGN;
  const int nscan = (int)((attn_len + SCAN_BLOCK - 1) / SCAN_BLOCK);
  if ((int64_t)nchunks + nscan > INT32_MAX) return TV_ERR_UNSUPPORTED;
  double* sums = static_cast<double*>(workspace);
  long long* firsts = reinterpret_cast<long long*>(sums + nchunks);
  int64_t* run_start = reinterpret_cast<int64_t*>(firsts + (int64_t)nscan * 3);
  int64_t* run_off = run_start + kMaxTopK;
  int* run_count = reinterpret_cast<int*>(run_off + kMaxTopK + 1);
  chunk_sums_kernel<<<nchunks + nscan, 256, 0, st>>>(attn, attn_len, starts, ends, nchunks, sums, firsts);
  int rc = check_launch();
  if (rc != TV_OK) return rc;
  chunk_select_kernel<<<1, SEL_THREADS, 0, st>>>(attn_len, starts, ends, nchunks, k, length, sums, firsts, nscan,
                                                 selected, run_start, run_off, run_count, max_indices, count, status);
  rc = check_launch();
  if (rc != TV_OK) return rc;
  const int64_t most = max_indices < length ? max_indices : length;   // the union never exceeds [0, length)
  if (most > 0) {
    expand_runs_kernel<<<(unsigned)((most + 255) / 256), 256, 0, st>>>(run_start, run_off, run_count, count,
                                                                       indices);
    rc = check_launch();
  }
  return rc;
}

int tv_gather_rows(int32_t planes, int32_t heads, const uint64_t* src, const uint64_t* dst,
                   int64_t src_head_stride_bytes, int64_t src_row_stride_bytes, int64_t dst_head_stride_bytes,
                   int64_t dst_row_stride_bytes, int32_t row_bytes, const int64_t* indices, const int64_t* count,
                   int64_t max_rows, void* stream) {
  if (planes < 0 || heads < 0 || max_rows < 0 || row_bytes < 0) return TV_ERR_SHAPE;
  if (planes == 0 || heads == 0 || max_rows == 0 || row_bytes == 0) return TV_OK;
  if (!src || !dst || !indices || !count) return TV_ERR_NULL;
  if ((row_bytes % 16) != 0 || (src_head_stride_bytes % 16) != 0 || (src_row_stride_bytes % 16) != 0 ||
      (dst_head_stride_bytes % 16) != 0 || (dst_row_stride_bytes % 16) != 0)
    return TV_ERR_ALIGN;
  if ((int64_t)planes * heads > 65535 || max_rows * (row_bytes / 16) > INT32_MAX) return TV_ERR_UNSUPPORTED;
  const int upr = row_bytes / 16;
  // enough threads for four units each at the largest count, spread over the SMs
  int64_t bx = (max_rows * upr + 4 * 256 - 1) / (4 * 256);
  const int64_t cap = ((int64_t)kNumSMs * 8 + planes * heads - 1) / (planes * heads);
  if (bx > cap) bx = cap;
  if (bx < 1) bx = 1;
  const dim3 grid((unsigned)bx, (unsigned)(planes * heads));
  gather_rows_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      heads, src, dst, src_head_stride_bytes, src_row_stride_bytes, dst_head_stride_bytes, dst_row_stride_bytes,
      upr, indices, count, max_rows);
  return check_launch();
}

}  // extern "C"
