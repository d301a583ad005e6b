// Sequence-sharded verify: the exchange of per-rank partials over NVLink peer
// memory (one process per GPU, buffers mapped into every rank).
//
// Each rank owns one buffer, mapped into every peer's address space:
//   [slot 0: O rows x D fp32 | lse rows fp32] [slot 1: same]
//   [flag 0, flag 1, ready, finished] [step counter]
// A step writes this rank's partial into slot s (the caller alternates s),
// then tv_peer_merge publishes flag[s] = step with a system-scope release,
// waits until every peer's flag[s] has reached the step, reads all ranks'
// partials with plain loads over NVLink and merges them by log-sum-exp in
// rank order -- every rank computes the same result.  A rank writes slot s again two steps later; by then every
// peer has passed the following step's wait, i.e. finished reading it, so the
// alternation needs no second barrier.  Waits are bounded (2 s): on expiry the
// merge records a status word and writes NaN rows.
#include "common.cuh"
#include "specverify.h"

namespace tv {
namespace {

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

struct PeerBases {
  const char* base[8];
};

template <typename T, int D, int W>
__global__ void __launch_bounds__(128) peer_merge_kernel(PeerBases pb, int world, int rank, int64_t slot_bytes,
                                                         int slot, int64_t flag_off, int* counter, int64_t rows,
                                                         void* out, float* out_lse, int* status) {
  constexpr int TPR = D / 4;          // threads per row, one float4 of O each
  constexpr int RPB = 128 / TPR;      // rows per block
  __shared__ int ok_s;
  // This rank's words at flag_off: [0..1] published step per slot (read by
  // peers over NVLink), [2] local "peers ready" word for the other blocks,
  // [3] blocks finished.  The step counter changes only at the very end of
  // the kernel, so every block derives the same step e from it.
  int* my_words = reinterpret_cast<int*>(const_cast<char*>(pb.base[rank]) + flag_off);
  const int e = *counter + 1;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long t0 = now_ns();
    if (blockIdx.x == 0) {
      // Publish this rank's partial (earlier launches on the stream wrote
      // it), then wait for every peer's; then release the other blocks.
      __threadfence_system();
      st_release_sys(my_words + slot, e);
      for (int p = 0; p < W && ok; ++p) {
        if (p == rank) continue;
        const int* flag = reinterpret_cast<const int*>(pb.base[p] + flag_off) + slot;
        unsigned it = 0;
        while (ld_acquire_sys(flag) < e) {
          if ((++it & 1023u) == 0 && now_ns() - t0 > 2000000000ull) {
            ok = 0;
            break;
          }
        }
      }
      if (!ok && status) atomicExch(status, 8);
      st_release_sys(my_words + 2, ok ? e : -e);
    } else {
      unsigned it = 0;
      for (;;) {
        const int w = ld_acquire_sys(my_words + 2);
        if (w == e) break;
        if (w == -e) {
          ok = 0;
          break;
        }
        if ((++it & 1023u) == 0 && now_ns() - t0 > 2000000000ull) {
          ok = 0;
          if (status) atomicExch(status, 8);
          break;
        }
      }
    }
    ok_s = ok;
  }
  __syncthreads();
  const int q = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * RPB + threadIdx.x / TPR;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  float lse = -INFINITY;
  if (row >= rows) {
  } else if (ok_s) {
    // All ranks' loads first (remote ones cross NVLink with ~us latency),
    // then the merge.
    float l[W];
    float4 v[W];
#pragma unroll
    for (int p = 0; p < W; ++p) {
      const float* part = reinterpret_cast<const float*>(pb.base[p] + slot * slot_bytes);
      l[p] = __ldcg(part + rows * D + row);
      v[p] = __ldcg(reinterpret_cast<const float4*>(part + row * D) + q);
    }
    float mx = -INFINITY;
#pragma unroll
    for (int p = 0; p < W; ++p) mx = fmaxf(mx, l[p]);
    float wsum = 0.f;
    if (mx != -INFINITY) {
#pragma unroll
      for (int p = 0; p < W; ++p) {
        const float w = l[p] == -INFINITY ? 0.f : expf(l[p] - mx);
        wsum += w;
        o[0] += w * v[p].x;
        o[1] += w * v[p].y;
        o[2] += w * v[p].z;
        o[3] += w * v[p].w;
      }
    }
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    for (int k = 0; k < 4; ++k) o[k] *= inv;
    lse = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  } else {
    for (int k = 0; k < 4; ++k) o[k] = __int_as_float(0x7fc00000);
    lse = __int_as_float(0x7fc00000);
  }
  if (row < rows) {
    T* dst = static_cast<T*>(out) + row * D + 4 * q;
    *reinterpret_cast<uint32_t*>(dst) = Elem<T>::pack2(o[0], o[1]);
    *reinterpret_cast<uint32_t*>(dst + 2) = Elem<T>::pack2(o[2], o[3]);
    if (q == 0 && out_lse) out_lse[row] = lse;
  }
  // The last block to finish advances the step counter (and resets the
  // finished-blocks word for the next step).
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(my_words + 3, 1) == (int)gridDim.x - 1) {
      my_words[3] = 0;
      *counter = e;
      __threadfence();
    }
  }
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" {

int tv_peer_merge(int32_t world, int32_t rank, const void* const* bases, int64_t slot_bytes, int32_t slot,
                  int64_t flag_offset, int32_t* counter, int64_t rows, int32_t head_dim, int32_t out_dtype,
                  void* out, float* out_lse, int32_t* status, void* stream) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return TV_ERR_SHAPE;
  if (!bases || !counter || !out) return TV_ERR_NULL;
  if (slot < 0 || slot > 1 || rows < 0) return TV_ERR_SHAPE;
  if (head_dim != 128 && head_dim != 64 && head_dim != 32) return TV_ERR_UNSUPPORTED;
  if ((slot_bytes % 16) != 0 || (flag_offset % 16) != 0) return TV_ERR_ALIGN;
  if (rows == 0) return TV_OK;
  PeerBases pb;
  for (int p = 0; p < 8; ++p) pb.base[p] = p < world ? static_cast<const char*>(bases[p]) : nullptr;
  for (int p = 0; p < world; ++p)
    if (!pb.base[p] || (reinterpret_cast<uintptr_t>(pb.base[p]) % 16) != 0) return TV_ERR_ALIGN;
  const int rpb = 128 / (head_dim / 4);
  dim3 grid((unsigned)((rows + rpb - 1) / rpb));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define TV_PEER_W(TT, DD, WW)                                                                              \
  peer_merge_kernel<TT, DD, WW><<<grid, 128, 0, st>>>(pb, world, rank, slot_bytes, slot, flag_offset, counter, \
                                                      rows, out, out_lse, status)
#define TV_PEER(TT, DD)                    \
  switch (world) {                         \
    case 1: TV_PEER_W(TT, DD, 1); break;   \
    case 2: TV_PEER_W(TT, DD, 2); break;   \
    case 3: TV_PEER_W(TT, DD, 3); break;   \
    case 4: TV_PEER_W(TT, DD, 4); break;   \
    case 5: TV_PEER_W(TT, DD, 5); break;   \
    case 6: TV_PEER_W(TT, DD, 6); break;   \
    case 7: TV_PEER_W(TT, DD, 7); break;   \
    default: TV_PEER_W(TT, DD, 8); break;  \
  }
  if (out_dtype == TV_BF16) {
    if (head_dim == 128) TV_PEER(__nv_bfloat16, 128)
    else if (head_dim == 64) TV_PEER(__nv_bfloat16, 64)
    else TV_PEER(__nv_bfloat16, 32)
  } else if (out_dtype == TV_F16) {
    if (head_dim == 128) TV_PEER(__half, 128)
    else if (head_dim == 64) TV_PEER(__half, 64)
    else TV_PEER(__half, 32)
  } else {
    return TV_ERR_DTYPE;
  }
#undef TV_PEER_W
#undef TV_PEER
  return check_launch();
}

}  // extern "C"
