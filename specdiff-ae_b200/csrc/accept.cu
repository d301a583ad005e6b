// Tree acceptance on the device.
//
// Stage 1 (grid rows x chunks): every CTA scans one slice of one node's
// vocabulary row with 16-byte loads and reduces (score, index) with the
// torch.argmax rule -- larger score wins, ties go to the smaller index, a NaN
// beats every number and the first NaN wins.  Greedy scores are the logits;
// sampling scores are logit / T + Gumbel noise, which makes the argmax an
// exact draw from softmax(logit / T).
//
// Stage 2 (one CTA): finishes the per-node argmax, then runs the acceptance
// rule of verify_new (diffspec/draft/tree_verification.py:120-182) entirely
// on the device: ok[i] = draft[i] == next[parent(i)], the synchronous
// ancestor closure, the first-maximum pick of the deepest accepted node, and
// the root-to-node path.  The reference copies parents, drafts and tokens to
// the host for this (tree_verification.py:112-118).
#include "accept_common.cuh"

namespace tv {
namespace {

using namespace acc;

constexpr int S1_THREADS = 256;
constexpr int S2_THREADS = 512;
constexpr int kMaxChunks = 64;

template <typename E>
__device__ __forceinline__ float to_float(E x);
template <> __device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_float<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_float<float>(float x) { return x; }

template <typename E, bool SAMPLE>
__global__ void __launch_bounds__(S1_THREADS) scan_kernel(const E* logits, int64_t sm, int vocab, int chunk,
                                                          float inv_t, uint64_t seed, uint64_t offset,
                                                          float* part_v, int* part_i) {
  const int row = blockIdx.x;
  const int ck = blockIdx.y;
  const int lo = ck * chunk;
  const int hi = min(vocab, lo + chunk);
  const E* src = logits + (int64_t)row * sm;
  Best b{-INFINITY, 0x7fffffff};
  constexpr int VEC = 16 / sizeof(E);
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(src + lo) & 15) == 0);
  int j0 = lo;
  if (vec_ok) {
    const int nvec = (hi - lo) / VEC;
    for (int v = threadIdx.x; v < nvec; v += S1_THREADS) {
      const int j = lo + v * VEC;
      const uint4 raw = *reinterpret_cast<const uint4*>(src + j);
      const E* e = reinterpret_cast<const E*>(&raw);
#pragma unroll
      for (int t = 0; t < VEC; ++t) {
        float x = to_float<E>(e[t]);
        if (SAMPLE) x = x * inv_t + gumbel(seed, offset, row, j + t);
        take(b, x, j + t);
      }
    }
    j0 = lo + nvec * VEC;
  }
  for (int j = j0 + threadIdx.x; j < hi; j += S1_THREADS) {
    float x = to_float<E>(src[j]);
    if (SAMPLE) x = x * inv_t + gumbel(seed, offset, row, j);
    take(b, x, j);
  }
  // Block reduction.
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float v = __shfl_xor_sync(0xffffffffu, b.v, o);
    const int i = __shfl_xor_sync(0xffffffffu, b.i, o);
    take(b, v, i);
  }
  __shared__ Best red[S1_THREADS / 32];
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = b;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < S1_THREADS / 32; ++w) take(b, red[w].v, red[w].i);
    part_v[row * gridDim.y + ck] = b.v;
    part_i[row * gridDim.y + ck] = b.i;
  }
}

__global__ void __launch_bounds__(S2_THREADS) decide_kernel(int rows, int chunks, const float* part_v,
                                                            const int* part_i, const int64_t* sampled,
                                                            const int64_t* draft, const int64_t* parent,
                                                            const int64_t* pos, int max_depth,
                                                            int64_t* next_tokens, int64_t* result,
                                                            const int* upstream_err) {
  extern __shared__ __align__(16) uint8_t sm[];
  int64_t* nxt = reinterpret_cast<int64_t*>(sm);                  // [rows]
  int* par = reinterpret_cast<int*>(nxt + rows);                   // [rows]
  uint8_t* ok = reinterpret_cast<uint8_t*>(par + rows);            // [rows]
  uint8_t* ok2 = ok + rows;                                        // [rows]
  __shared__ int bad;
  __shared__ int64_t red_v[S2_THREADS / 32];
  __shared__ int red_i[S2_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (upstream_err && *upstream_err != 0) {   // the partials are not valid
    for (int i = tid; i < rows; i += S2_THREADS) next_tokens[i] = -1;
    if (tid == 0 && result) {
      result[0] = TV_ERR_LAUNCH;
      for (int k = 1; k < 8; ++k) result[k] = 0;
    }
    return;
  }
  if (tid == 0) bad = 0;

  // 1. per-node target token
  for (int i = warp; i < rows; i += S2_THREADS / 32) {
    int64_t tok;
    if (sampled) {
      tok = sampled[i];
    } else {
      // all of a lane's partials are loaded before they are compared, so the
      // loads overlap instead of waiting one by one
      Best b{-INFINITY, 0x7fffffff};
      for (int c0 = 0; c0 < chunks; c0 += 32 * 8) {
        float v[8];
        int ix[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int c = c0 + u * 32 + lane;
          v[u] = c < chunks ? part_v[i * chunks + c] : -INFINITY;
          ix[u] = c < chunks ? part_i[i * chunks + c] : 0x7fffffff;
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) take(b, v[u], ix[u]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, b.v, o);
        const int ix = __shfl_xor_sync(0xffffffffu, b.i, o);
        take(b, v, ix);
      }
      tok = b.i;
    }
    if (lane == 0) {
      nxt[i] = tok;
      next_tokens[i] = tok;
    }
  }
  if (!draft) return;   // next tokens only (uniform across the CTA)
  __syncthreads();

  // 2. parents over all rows (tree_verification.py:120-125) and first test
  for (int i = tid; i < rows; i += S2_THREADS) {
    int pe = 0;
    if (i > 0) {
      int64_t pr = parent[i - 1];
      if (pr == i - 1) pr = -1;
      if (pr < -1 || pr >= rows - 1) {
        bad = 1;
        pr = -1;
      }
      pe = (int)pr + 1;
    }
    par[i] = pe;
  }
  __syncthreads();
  for (int i = tid; i < rows; i += S2_THREADS) ok[i] = (i == 0) || (draft[i] == nxt[par[i]]);
  __syncthreads();

  // 3. synchronous closure, at most min(max_depth + 2, rows) rounds
  const int hops = min(max_depth + 2, rows);
  for (int hgo = 0; hgo < hops; ++hgo) {
    int changed = 0;
    for (int i = tid; i < rows; i += S2_THREADS) {
      const uint8_t v = ok[i] & ok[par[i]];
      ok2[i] = v;
      changed |= (v != ok[i]);
    }
    changed = __syncthreads_or(changed);
    if (!changed) break;
    for (int i = tid; i < rows; i += S2_THREADS) ok[i] = ok2[i];
    __syncthreads();
  }

  // 4. deepest accepted node: first maximum of (ok ? pos : 0)
  int64_t bv = INT64_MIN;
  int bi = 0x7fffffff;
  for (int i = tid; i < rows; i += S2_THREADS) {
    const int64_t v = ok[i] ? pos[i] : 0;
    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int64_t v = __shfl_xor_sync(0xffffffffu, bv, o);
    const int ix = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v > bv || (v == bv && ix < bi)) { bv = v; bi = ix; }
  }
  if (lane == 0) { red_v[warp] = bv; red_i[warp] = bi; }
  __syncthreads();

  // 5. path root -> best (thread 0; at most `rows` steps)
  if (tid == 0) {
    for (int w = 1; w < S2_THREADS / 32; ++w)
      if (red_v[w] > bv || (red_v[w] == bv && red_i[w] < bi)) { bv = red_v[w]; bi = red_i[w]; }
    const int best = bi;
    int64_t* ids = result + 8;
    int64_t* toks = result + 8 + rows;
    int n = 0;
    int cur = best;
    int status = bad ? TV_ERR_INPUT : TV_OK;
    while (cur != -1) {
      if (n >= rows) { status = TV_ERR_INPUT; break; }  // parent pointers form a cycle
      ids[n++] = cur;
      cur = cur == 0 ? -1 : par[cur];
    }
    for (int a = 0, z = n - 1; a < z; ++a, --z) {
      const int64_t t = ids[a]; ids[a] = ids[z]; ids[z] = t;
    }
    for (int j = 0; j < n; ++j) toks[j] = draft[ids[j]];
    result[0] = status;
    result[1] = best;
    result[2] = n;
    result[3] = nxt[best];
    result[4] = result[5] = result[6] = result[7] = 0;
  }
}

}  // namespace

int launch_accept_decide(int rows, int chunks, const float* part_v, const int* part_i, const int64_t* sampled,
                         const int64_t* draft, const int64_t* parent, const int64_t* pos, int max_depth,
                         int64_t* next_tokens, int64_t* result, const int* upstream_err, cudaStream_t st) {
  const size_t smem = (size_t)rows * (sizeof(int64_t) + sizeof(int) + 2);
  if (smem > 200 * 1024) return TV_ERR_UNSUPPORTED;
  if (smem > 48 * 1024) {
    const int rc_smem = ensure_dynamic_smem(reinterpret_cast<const void*>(decide_kernel), (int)smem);
    if (rc_smem != TV_OK) return rc_smem;
  }
  decide_kernel<<<1, S2_THREADS, smem, st>>>(rows, chunks, part_v, part_i, sampled, draft, parent, pos, max_depth,
                                             next_tokens, result, upstream_err);
  return check_launch();
}

namespace {

int choose_chunks(int rows, int vocab) {
  int c = (2 * kNumSMs + rows - 1) / rows;
  const int max_by_size = (vocab + 2047) / 2048;
  if (c > max_by_size) c = max_by_size;
  if (c > kMaxChunks) c = kMaxChunks;
  return c < 1 ? 1 : c;
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" {

int tv_accept_workspace_size(const tv_accept_args* a, size_t* bytes) {
  if (!a || !bytes) return TV_ERR_NULL;
  const int chunks = choose_chunks(a->rows > 0 ? a->rows : 1, a->vocab > 0 ? a->vocab : 1);
  *bytes = (size_t)(a->rows > 0 ? a->rows : 0) * chunks * (sizeof(float) + sizeof(int)) + 64;
  return TV_OK;
}

int tv_accept(const tv_accept_args* a, void* stream) {
  if (!a) return TV_ERR_NULL;
  if (a->mode < 0 || a->mode > 2) return TV_ERR_INPUT;
  if (a->rows <= 0 || a->max_depth < 0) return TV_ERR_SHAPE;
  if (a->rows > 8192) return TV_ERR_UNSUPPORTED;
  if (!a->draft || !a->pos || !a->next_tokens || !a->result) return TV_ERR_NULL;
  if (a->rows > 1 && !a->parent) return TV_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rows = a->rows;
  int chunks = 1;
  float* pv = nullptr;
  int* pi = nullptr;
  if (a->mode != 2) {
    if (!a->logits) return TV_ERR_NULL;
    if (a->vocab <= 0) return TV_ERR_SHAPE;
    if (a->mode == 1 && !(a->temperature > 0.f)) return TV_ERR_INPUT;
    chunks = choose_chunks(rows, a->vocab);
    size_t need = 0;
    tv_accept_workspace_size(a, &need);
    if (!a->workspace || a->workspace_bytes < need) return TV_ERR_WORKSPACE;
    if ((reinterpret_cast<uintptr_t>(a->workspace) & 15) != 0) return TV_ERR_ALIGN;
    pv = static_cast<float*>(a->workspace);
    pi = reinterpret_cast<int*>(pv + (size_t)rows * chunks);
    int chunk = (a->vocab + chunks - 1) / chunks;
    chunk = (chunk + 7) & ~7;
    chunks = (a->vocab + chunk - 1) / chunk;
    dim3 grid(rows, chunks);
    const float inv_t = a->mode == 1 ? 1.0f / a->temperature : 1.0f;
    const bool s = a->mode == 1;
    switch (a->logits_dtype) {
      case TV_BF16:
        if (s) scan_kernel<__nv_bfloat16, true><<<grid, S1_THREADS, 0, st>>>(static_cast<const __nv_bfloat16*>(a->logits), a->logits_sm, a->vocab, chunk, inv_t, a->seed, a->offset, pv, pi);
        else scan_kernel<__nv_bfloat16, false><<<grid, S1_THREADS, 0, st>>>(static_cast<const __nv_bfloat16*>(a->logits), a->logits_sm, a->vocab, chunk, inv_t, a->seed, a->offset, pv, pi);
        break;
      case TV_F16:
        if (s) scan_kernel<__half, true><<<grid, S1_THREADS, 0, st>>>(static_cast<const __half*>(a->logits), a->logits_sm, a->vocab, chunk, inv_t, a->seed, a->offset, pv, pi);
        else scan_kernel<__half, false><<<grid, S1_THREADS, 0, st>>>(static_cast<const __half*>(a->logits), a->logits_sm, a->vocab, chunk, inv_t, a->seed, a->offset, pv, pi);
        break;
      case TV_F32:
        if (s) scan_kernel<float, true><<<grid, S1_THREADS, 0, st>>>(static_cast<const float*>(a->logits), a->logits_sm, a->vocab, chunk, inv_t, a->seed, a->offset, pv, pi);
        else scan_kernel<float, false><<<grid, S1_THREADS, 0, st>>>(static_cast<const float*>(a->logits), a->logits_sm, a->vocab, chunk, inv_t, a->seed, a->offset, pv, pi);
        break;
      default: return TV_ERR_DTYPE;
    }
    const int rc = check_launch();
    if (rc != TV_OK) return rc;
  } else if (!a->sampled) {
    return TV_ERR_NULL;
  }
  return launch_accept_decide(rows, chunks, pv, pi, a->mode == 2 ? a->sampled : nullptr, a->draft, a->parent, a->pos,
                              a->max_depth, a->next_tokens, a->result, nullptr, st);
}

}  // extern "C"
