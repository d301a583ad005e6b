// Sequence-sharded verify: the exchange of per-rank partials over NVLink peer
// memory, fused with the combine of this rank's split-KV partials and the
// final merge (one kernel after the attention kernel, one process per GPU).
//
// Each rank owns one exchange buffer, mapped into every rank's address space
// (rows = B * H * M query rows, in the attention kernel's row order
// (b, kv head, node, group member); D = head_dim; W = world size):
//   slot s (s = 0, 1) at s * slot_bytes:
//     O   [W][rows][D] fp32        -- rank r's partial at r * rows * D
//     LSE [W][rows] fp32
//     final O [rows][D] fp32, final LSE [rows]   (owner mode)
//   flags at flags_off: int32 [2][W][row blocks]   "partial arrived"
//         at fin_flags_off: int32 [2][row blocks]  "final rows arrived"
//   then two int32 words: [steps completed, blocks finished this step]
// all zero before the first step.
//
// Step e (1, 2, ...) uses slot e & 1.  Each block takes row blocks of RPB rows
// and combines this rank's split partials of those rows (local memory).  Two
// exchange modes:
//  * push to all (default): the block stores its rows into every
//    peer's slot region for this rank (posted NVLink writes), publishes
//    flags[slot][rank][row block] = e on each peer with a system-scope
//    release, waits -- on its own, local flags -- until every peer has
//    published the same row block, and merges all W partials by log-sum-exp
//    in rank order.  One NVLink hop; (W - 1) x the partial leaves each rank.
//  * owner (on request): row block rb belongs to rank rb * W / nrb.
//    Every other rank pushes its partial rows of rb to the owner only; the
//    owner merges them in rank order and pushes the final fp32 rows to every
//    other rank, which convert them exactly as the owner does.  Two hops, but
//    about 2 x (W - 1) / W of one partial leaves each rank instead of W - 1.
// Either way every rank computes bit-identical outputs and no block waits on
// more than the row block it is working on.
//
// Slot reuse: a region of slot s written by a remote rank at step e + 2 was
// last read by its owner at step e.  The writer reaches step e + 2 only after
// its step e + 1 kernel finished, which waited for a step e + 1 flag that the
// reader raises only in its step e + 1 kernel (in owner mode the final rows
// wait for the partials' flags of the same step and vice versa), and that
// kernel starts after the reader's step e kernel completed.  So two slots
// need no second handshake.  Waits are bounded (2 s per launch): on expiry
// the status word gets 8 and the rows affected are NaN.
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
  int64_t lse_off;       // partials' LSE array inside a slot
  int64_t fin_off;       // final O inside a slot
  int64_t fin_lse_off;   // final LSE inside a slot
  int64_t slot_bytes;
  int64_t flags_off;     // int32 [2][W][nrb]
  int64_t fin_flags_off; // int32 [2][nrb]
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
  L.fin_off = L.lse_off + align256((int64_t)world * rows * 4);
  L.fin_lse_off = L.fin_off + align256(rows * D * 4);
  L.slot_bytes = L.fin_lse_off + align256(rows * 4);
  L.flags_off = 2 * L.slot_bytes;
  L.fin_flags_off = L.flags_off + align256((int64_t)2 * world * L.nrb * 4);
  L.words_off = L.fin_flags_off + align256((int64_t)2 * L.nrb * 4);
  L.total = L.words_off + 256;
  return L;
}

struct PeerBases {
  char* base[kMaxPeers];
};

// Log-sum-exp merge of W normalised partials in rank order.
template <int W>
__device__ __forceinline__ void merge_ranks(const float (&l)[W], const float4 (&v)[W], float4& o, float& lse) {
  float mx = -INFINITY;
#pragma unroll
  for (int pr = 0; pr < W; ++pr) mx = fmaxf(mx, l[pr]);
  float wsum = 0.f;
  o = make_float4(0.f, 0.f, 0.f, 0.f);
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
  lse = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
  o = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
}

// Bounded wait until *flag >= e; false once the launch's deadline passed.
__device__ __forceinline__ bool wait_flag(const int* flag, int e, unsigned long long deadline) {
  unsigned it = 0;
  while (ld_acquire_sys(flag) < e) {
    if ((++it & 255u) == 0 && now_ns() > deadline) return false;
  }
  return true;
}

template <typename T, int D, int W, bool OWNED>
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
  const float nan = __int_as_float(0x7fc00000);
  // flags[slot][src][rb] and fin_flags[slot][rb] of the buffer at `base`
  auto part_flag = [&](char* base, int src, int rb) {
    return reinterpret_cast<int*>(base + L.flags_off) + ((int64_t)slot * W + src) * L.nrb + rb;
  };
  auto fin_flag = [&](char* base, int rb) {
    return reinterpret_cast<int*>(base + L.fin_flags_off) + (int64_t)slot * L.nrb + rb;
  };
  for (int rb = blockIdx.x; rb < L.nrb; rb += gridDim.x) {
    const int64_t row = (int64_t)rb * RPB + threadIdx.x / TPR;
    const bool valid = row < L.rows;
    const int owner = OWNED ? (int)((int64_t)rb * W / L.nrb) : rank;
    int bh = 0, r = 0;
    float4 own = make_float4(0.f, 0.f, 0.f, 0.f);
    float own_l = -INFINITY;
    if (valid) {
      bh = (int)(row / p.R);
      r = (int)(row - (int64_t)bh * p.R);
      combine_split_row<D>(p, bh, r, q, own, own_l);
#pragma unroll
      for (int pr = 0; pr < W; ++pr) {
        if (pr == rank || (OWNED && pr != owner)) continue;
        char* dst = pb.base[pr] + slot_off;
        reinterpret_cast<float4*>(dst)[((int64_t)rank * L.rows + row) * TPR + q] = own;
        if (q == 0) reinterpret_cast<float*>(dst + L.lse_off)[(int64_t)rank * L.rows + row] = own_l;
      }
    }
    __syncthreads();   // the block's pushes precede each flag's release
    int ok = 1;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    float lse = -INFINITY;
    if (owner == rank) {
      if (t < W && t != rank) {
        if (!OWNED) {
          __threadfence_system();
          st_release_sys(part_flag(pb.base[t], rank, rb), e);
        }
        ok = wait_flag(part_flag(mine, t, rb), e, deadline);
      }
      ok = __syncthreads_and(ok);
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
        merge_ranks<W>(l, v, o, lse);
        if (!ok) {
          o = make_float4(nan, nan, nan, nan);
          lse = nan;
        }
      }
      if (OWNED) {
        // Hand the final rows to every other rank.
        if (valid) {
#pragma unroll
          for (int pr = 0; pr < W; ++pr) {
            if (pr == rank) continue;
            char* dst = pb.base[pr] + slot_off;
            reinterpret_cast<float4*>(dst + L.fin_off)[row * TPR + q] = o;
            if (q == 0) reinterpret_cast<float*>(dst + L.fin_lse_off)[row] = lse;
          }
        }
        __syncthreads();
        if (t < W && t != rank) {
          __threadfence_system();
          st_release_sys(fin_flag(pb.base[t], rb), e);
        }
      }
    } else {
      // Owner mode, a row block of another rank: publish the partial to the
      // owner, then wait for its final rows.
      if (t == 0) {
        __threadfence_system();
        st_release_sys(part_flag(pb.base[owner], rank, rb), e);
        ok = wait_flag(fin_flag(mine, rb), e, deadline);
      }
      ok = __syncthreads_and(ok);
      if (valid) {
        const char* src = mine + slot_off;
        o = __ldcg(reinterpret_cast<const float4*>(src + L.fin_off) + row * TPR + q);
        lse = __ldcg(reinterpret_cast<const float*>(src + L.fin_lse_off) + row);
        if (!ok) {
          o = make_float4(nan, nan, nan, nan);
          lse = nan;
        }
      }
    }
    if (!ok && t == 0 && p.err) atomicExch(p.err, 8);
    if (valid) {
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

template <typename T, int D, bool OWNED>
void launch_w(int world, dim3 grid, const AttnParams& p, const PeerBases& pb, int rank, const ExLayout& L,
              cudaStream_t st) {
  switch (world) {
    case 1: sharded_combine_kernel<T, D, 1, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 2: sharded_combine_kernel<T, D, 2, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 3: sharded_combine_kernel<T, D, 3, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 4: sharded_combine_kernel<T, D, 4, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 5: sharded_combine_kernel<T, D, 5, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 6: sharded_combine_kernel<T, D, 6, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    case 7: sharded_combine_kernel<T, D, 7, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
    default: sharded_combine_kernel<T, D, 8, OWNED><<<grid, kThreads, 0, st>>>(p, pb, rank, L); break;
  }
}

template <typename T, bool OWNED>
void launch_t(int D, int world, dim3 grid, const AttnParams& p, const PeerBases& pb, int rank, const ExLayout& L,
              cudaStream_t st) {
  if (D == 128) launch_w<T, 128, OWNED>(world, grid, p, pb, rank, L, st);
  else if (D == 64) launch_w<T, 64, OWNED>(world, grid, p, pb, rank, L, st);
  else launch_w<T, 32, OWNED>(world, grid, p, pb, rank, L, st);
}

}  // namespace

int launch_sharded_combine(const AttnParams& p, int dtype, int D, int world, int rank, const void* const* bases,
                           bool owned, cudaStream_t st) {
  const ExLayout L = layout(world, (int64_t)p.B * p.Hkv * p.R, D);
  PeerBases pb;
  for (int r = 0; r < kMaxPeers; ++r) pb.base[r] = r < world ? static_cast<char*>(const_cast<void*>(bases[r])) : nullptr;
  // Every block of the grid must be resident at once (a block waits for the
  // peers' blocks of the same row blocks): at most 4 blocks of 128 threads
  // per SM, each looping over row blocks.
  const int grid = L.nrb < 4 * kNumSMs ? L.nrb : 4 * kNumSMs;
  owned = owned && world > 1;
  if (dtype == TV_BF16) {
    if (owned) launch_t<__nv_bfloat16, true>(D, world, dim3(grid), p, pb, rank, L, st);
    else launch_t<__nv_bfloat16, false>(D, world, dim3(grid), p, pb, rank, L, st);
  } else {
    if (owned) launch_t<__half, true>(D, world, dim3(grid), p, pb, rank, L, st);
    else launch_t<__half, false>(D, world, dim3(grid), p, pb, rank, L, st);
  }
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
