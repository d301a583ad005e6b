// Sequence-sharded verify: the exchange of per-rank partials over NVLink peer
// memory, fused with the combine of this rank's split-KV partials and the
// final merge (one kernel after the attention kernel, one process per GPU).
//
// Each rank owns one exchange buffer, mapped into every rank's address space
// (rows = B * H * M query rows, in the attention kernel's row order
// (b, kv head, node, group member); D = head_dim; W = world size):
//   slot s (s = 0, 1) at s * slot_bytes:
//     O   [W][rows][D] fp32        -- rank r's partial at r * rows * D
//     LSE [W][rows] fp32           -- at byte lse_off of the slot
//   flags at 2 * slot_bytes: int32 [2][W][row blocks]
//   then two int32 words: [steps completed, blocks finished this step]
// all zero before the first step.
//
// Step e (1, 2, ...) uses slot e & 1.  Each block takes row blocks of RPB rows:
// it combines this rank's split partials of those rows (local memory), stores
// the result into every peer's slot region for this rank (posted NVLink
// writes), then publishes flags[slot][rank][row block] = e on each peer with a
// system-scope release.  It then waits -- on its own, local flags -- until
// every peer has published the same row block, reads the peers' rows from its
// own buffer and merges all W partials by log-sum-exp in rank order, so every
// rank computes bit-identical outputs.  Nothing waits on more than the one
// row block it merges.
//
// Slot reuse: rank r overwrites its region of slot s on peer p at step e + 2.
// Step e + 2 runs after r's step e + 1 kernel finished, which waited for
// every row block of p's step e + 1 publication; p's step e + 1 kernel starts
// only after its step e kernel -- the one that read slot s -- completed.  So
// two slots need no second handshake.  Waits are bounded (2 s per launch):
// on expiry the status word gets 8 and the rows affected are NaN.
#include "attn_epilogue.cuh"
#include "attn_kernels.cuh"
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

constexpr int kThreads = 128;

// Byte offsets inside one rank's exchange buffer.
struct ExLayout {
  int64_t rows;          // query rows of one partial
  int64_t lse_off;       // LSE array inside a slot
  int64_t slot_bytes;
  int64_t flags_off;     // int32 [2][W][nrb]
  int64_t words_off;     // int32 [steps completed, blocks finished]
  int64_t total;
  int nrb;               // row blocks
};

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

ExLayout layout(int world, int64_t rows, int D) {
  ExLayout L;
  const int rpb = kThreads / (D / 4);
  L.rows = rows;
  L.nrb = (int)((rows + rpb - 1) / rpb);
  L.lse_off = align256((int64_t)world * rows * D * 4);
  L.slot_bytes = L.lse_off + align256((int64_t)world * rows * 4);
  L.flags_off = 2 * L.slot_bytes;
  L.words_off = L.flags_off + align256((int64_t)2 * world * L.nrb * 4);
  L.total = L.words_off + 256;
  return L;
}

struct PeerBases {
  char* base[kMaxPeers];
};

template <typename T, int D, int W>
__global__ void __launch_bounds__(kThreads, 4)
    sharded_combine_kernel(const AttnParams p, const PeerBases pb, int rank, const ExLayout L) {
  constexpr int TPR = D / 4;            // threads per row, one float4 of O each
  constexpr int RPB = kThreads / TPR;   // rows per row block
  char* const mine = pb.base[rank];
  int* const words = reinterpret_cast<int*>(mine + L.words_off);
  // Every block reads the step count before any block can advance it (the
  // last block to finish does, below).
  const int e = *reinterpret_cast<volatile int*>(words) + 1;
  const int slot = e & 1;
  const int64_t slot_off = slot * L.slot_bytes;
  const unsigned long long deadline = now_ns() + 2000000000ull;
  const int q = threadIdx.x % TPR;
  const int t = threadIdx.x;
  for (int rb = blockIdx.x; rb < L.nrb; rb += gridDim.x) {
    const int64_t row = (int64_t)rb * RPB + threadIdx.x / TPR;
    const bool valid = row < L.rows;
    int bh = 0, r = 0;
    float4 own = make_float4(0.f, 0.f, 0.f, 0.f);
    float own_l = -INFINITY;
    if (valid) {
      bh = (int)(row / p.R);
      r = (int)(row - (int64_t)bh * p.R);
      combine_split_row<D>(p, bh, r, q, own, own_l);
#pragma unroll
      for (int pr = 0; pr < W; ++pr) {
        if (pr == rank) continue;
        char* dst = pb.base[pr] + slot_off;
        reinterpret_cast<float4*>(dst)[((int64_t)rank * L.rows + row) * TPR + q] = own;
        if (q == 0) reinterpret_cast<float*>(dst + L.lse_off)[(int64_t)rank * L.rows + row] = own_l;
      }
    }
    __syncthreads();   // the block's pushes precede each flag's release
    int ok = 1;
    if (t < W && t != rank) {
      __threadfence_system();
      st_release_sys(reinterpret_cast<int*>(pb.base[t] + L.flags_off) + ((int64_t)slot * W + rank) * L.nrb + rb, e);
      const int* flag = reinterpret_cast<const int*>(mine + L.flags_off) + ((int64_t)slot * W + t) * L.nrb + rb;
      unsigned it = 0;
      while (ld_acquire_sys(flag) < e) {
        if ((++it & 255u) == 0 && now_ns() > deadline) {
          ok = 0;
          break;
        }
      }
    }
    ok = __syncthreads_and(ok);
    if (!ok && t == 0 && p.err) atomicExch(p.err, 8);
    if (valid) {
      float l[W];
      float4 v[W];
      const char* src = mine + slot_off;
#pragma unroll
      for (int pr = 0; pr < W; ++pr) {
        if (pr == rank) {
          l[pr] = own_l;
          v[pr] = own;
        } else {
          l[pr] = __ldcg(reinterpret_cast<const float*>(src + L.lse_off) + (int64_t)pr * L.rows + row);
          v[pr] = __ldcg(reinterpret_cast<const float4*>(src) + ((int64_t)pr * L.rows + row) * TPR + q);
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int pr = 0; pr < W; ++pr) mx = fmaxf(mx, l[pr]);
      float wsum = 0.f;
      float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
      if (mx != -INFINITY) {
#pragma unroll
        for (int pr = 0; pr < W; ++pr) {
          const float w = l[pr] == -INFINITY ? 0.f : expf(l[pr] - mx);
          wsum += w;
          o.x += w * v[pr].x;
          o.y += w * v[pr].y;
          o.z += w * v[pr].z;
          o.w += w * v[pr].w;
        }
      }
      const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
      float lse = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
      o = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
      if (!ok) {
        const float nan = __int_as_float(0x7fc00000);
        o = make_float4(nan, nan, nan, nan);
        lse = nan;
      }
      const int b = bh / p.Hkv;
      const int hk = bh - b * p.Hkv;
      int m, h;
      row_coords(p, hk, r, m, h);
      store_out_pair<T>(p, b, m, h, 4 * q, o.x, o.y);
      store_out_pair<T>(p, b, m, h, 4 * q + 2, o.z, o.w);
      if (q == 0) store_row_stats<T>(p, b, m, h, lse);
    }
  }
  // The last block to finish advances the step count and resets the
  // finished-blocks word for the next step.
  __syncthreads();
  if (t == 0) {
    __threadfence();
    if (atomicAdd(words + 1, 1) == (int)gridDim.x - 1) {
      words[1] = 0;
      words[0] = e;
      __threadfence();
    }
  }
}

template <typename T, int D>
void launch_w(int world, dim3 grid, const AttnParams& p, const PeerBases& pb, int rank, const ExLayout& L,
              cudaStream_t st) {
  switch (world) {
    case 1: sharded_combine_kernel<T, D, 1><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 2: sharded_combine_kernel<T, D, 2><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 3: sharded_combine_kernel<T, D, 3><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 4: sharded_combine_kernel<T, D, 4><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 5: sharded_combine_kernel<T, D, 5><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 6: sharded_combine_kernel<T, D, 6><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 7: sharded_combine_kernel<T, D, 7><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    default: sharded_combine_kernel<T, D, 8><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
  }
}

template <typename T>
void launch_t(int D, int world, dim3 grid, const AttnParams& p, const PeerBases& pb, int rank, const ExLayout& L,
              cudaStream_t st) {
  if (D == 128) launch_w<T, 128>(world, grid, p, pb, rank, L, st);
  else if (D == 64) launch_w<T, 64>(world, grid, p, pb, rank, L, st);
  else launch_w<T, 32>(world, grid, p, pb, rank, L, st);
}

}  // namespace

int launch_sharded_combine(const AttnParams& p, int dtype, int D, int world, int rank, const void* const* bases,
                           cudaStream_t st) {
  const ExLayout L = layout(world, (int64_t)p.B * p.Hkv * p.R, D);
  PeerBases pb;
  for (int r = 0; r < kMaxPeers; ++r) pb.base[r] = r < world ? static_cast<char*>(const_cast<void*>(bases[r])) : nullptr;
  // Every block of the grid must be resident at once (a block waits for the
  // peers' blocks of the same row blocks): at most 4 blocks of 128 threads
  // per SM, each looping over row blocks.
  const int grid = L.nrb < 4 * kNumSMs ? L.nrb : 4 * kNumSMs;
  if (dtype == TV_BF16) launch_t<__nv_bfloat16>(D, world, dim3(grid), p, pb, rank, L, st);
  else launch_t<__half>(D, world, dim3(grid), p, pb, rank, L, st);
  return check_launch();
}

}  // namespace tv

using namespace tv;

extern "C" int tv_sharded_exchange_bytes(int32_t world, int64_t rows, int32_t head_dim, int64_t* bytes) {
  if (!bytes) return TV_ERR_NULL;
  *bytes = 0;
  if (world < 1 || world > kMaxPeers || rows < 0) return TV_ERR_SHAPE;
  if (head_dim != 128 && head_dim != 64 && head_dim != 32) return TV_ERR_UNSUPPORTED;
  *bytes = layout(world, rows, head_dim).total;
  return TV_OK;
}
