// Sequence-sharded verify: the exchange of per-rank partials over NVLink peer
// memory, fused with the combine of this rank's split-KV partials and the
// final merge (one kernel after the attention kernel, one process per GPU).
//
// Every value crosses NVLink as an 8-byte word: the fp32 bits in the low
// half, the step number e in the high half.  An aligned 64-bit store is
// single-copy atomic, so a reader that sees step e in a word also sees that
// step's value: no flags, no fences.  A reader accepts step e exactly: a word
// of a later step means a peer that already gave up on this rank (a timed-out
// wait) has moved on and overwritten the slot, so this rank flags the row
// (status 8, NaN) instead of merging another step's values.
// (System-scope fence + flag pairs, one per block, measured ~15 us per step
// on B200 even with no peer to wait for; the words double the bytes instead,
// ~1 us per MB at NVLink rates.)
//
// Each rank owns one exchange buffer, mapped into every rank's address space
// (rows = B * H * M query rows, in the attention kernel's row order
// (b, kv head, node, group member); D = head_dim; W = world size):
//   slot s (s = 0, 1) at s * slot_bytes, all 8-byte words:
//     O   [W][rows][D]      -- rank r's partial at r * rows * D
//     LSE [W][rows]
//     final O [rows][D], final LSE [rows]   (owner mode; with a 16-bit
//         output the final O words carry two values each: [rows][D / 2])
//   then int32 step counts, one per block of the kernel's grid
// all zero before the first step.
//
// Step e (1, 2, ...) uses slot e & 1.  Each block takes row blocks of RPB rows
// and combines this rank's split partials of those rows (local memory),
// keeping the result in its own rank's region of its own buffer (only this
// rank writes there).  Two exchange modes:
//  * push to all (default below 4 ranks): the block stores its rows into
//    every peer's slot region for this rank, then waits on its own buffer
//    until every peer's words of the same rows carry step e, and merges all
//    W partials by log-sum-exp in rank order.  One hop; 2 (W - 1) x the
//    fp32 partial leaves each rank.
//  * owner (default from 4 ranks on): row block rb belongs to rank
//    rb * W / nrb.  The other ranks push their partial rows of rb to the owner
//    only; the owner merges them in rank order and pushes the final rows to
//    every other rank -- in the output type (two 16-bit values per word, or
//    fp32 words for an fp32 output), so every rank writes what the owner
//    writes.  Two hops, but about 3 (W - 1) / W partials' worth of words
//    leave each rank instead of 2 (W - 1).
// Either way every rank computes bit-identical outputs and no thread waits on
// more than the rows it is working on.
//
// Slot reuse: a region of slot s written by a remote rank at step e + 2 was
// last read by its owner at step e.  The writer reaches step e + 2 only after
// its step e + 1 kernel finished, and that kernel waited for words the reader
// wrote in its own step e + 1 kernel (push: the reader's partial; owner mode:
// the final rows, or the partial that the final rows' owner waited for),
// which starts after the reader's step e kernel completed.  So two slots need
// no second handshake -- as long as every wait succeeds.  Waits are bounded
// (2 s per launch): on expiry the status word gets 8 and the rows affected
// are NaN; the rank then runs ahead of a lagging peer, which sees the later
// step's tags and flags its rows the same way.
#include "attn_epilogue.cuh"
#include "attn_kernels.cuh"
#include "common.cuh"
#include "specverify.h"

namespace tv {
namespace {

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

constexpr int kThreads = 128;
// Blocks per SM of the exchange kernel (its registers allow) -- the grid is
// capped so that all blocks are resident at once: a thread waits for words
// that the peers' blocks of the same index write.
constexpr int blocks_per_sm(int world) { return world > 4 ? 3 : 4; }
constexpr int kMaxGrid = 4 * kNumSMs;

using u64 = unsigned long long;

// Byte offsets inside one rank's exchange buffer.
struct ExLayout {
  int64_t rows;          // query rows of one partial
  int64_t lse_off;       // partials' LSE words inside a slot
  int64_t fin_off;       // final O words inside a slot
  int64_t fin_lse_off;   // final LSE words inside a slot
  int64_t slot_bytes;
  int64_t steps_off;     // int32 step count per block
  int64_t total;
  int nrb;               // row blocks
};

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

ExLayout layout(int world, int64_t rows, int D) {
  ExLayout L;
  const int rpb = kThreads / (D / 4);
  L.rows = rows;
  L.nrb = (int)((rows + rpb - 1) / rpb);
  L.lse_off = align256((int64_t)world * rows * D * 8);
  L.fin_off = L.lse_off + align256((int64_t)world * rows * 8);
  L.fin_lse_off = L.fin_off + align256(rows * D * 8);
  L.slot_bytes = L.fin_lse_off + align256(rows * 8);
  L.steps_off = 2 * L.slot_bytes;
  L.total = L.steps_off + align256(4 * kMaxGrid);
  return L;
}

__device__ __forceinline__ u64 ll_word(float v, int e) {
  return ((u64)(unsigned)e << 32) | __float_as_uint(v);
}
// Four values of step e at dst (32-byte aligned), as two 16-byte stores of
// two single-copy-atomic words each.
__device__ __forceinline__ void ll_put4(u64* dst, float4 v, int e) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(ll_word(v.x, e)), "l"(ll_word(v.y, e))
               : "memory");
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + 2), "l"(ll_word(v.z, e)), "l"(ll_word(v.w, e))
               : "memory");
}
__device__ __forceinline__ void ll_put1(u64* dst, float v, int e) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(dst), "l"(ll_word(v, e)) : "memory");
}
// Bounded waits until the words carry step e.  False once the launch's
// deadline has passed, or at once when a word carries a later step (this
// rank fell behind a peer that timed out on it: step e's values are gone).
__device__ __forceinline__ bool ll_get4(const u64* src, int e, unsigned long long deadline, float4& v) {
  unsigned it = 0;
  for (;;) {
    u64 a, b, c, d;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(c), "=l"(d) : "l"(src + 2) : "memory");
    const int ta = (int)(a >> 32), tb = (int)(b >> 32), tc = (int)(c >> 32), td = (int)(d >> 32);
    if (ta == e && tb == e && tc == e && td == e) {
      v = make_float4(__uint_as_float((unsigned)a), __uint_as_float((unsigned)b), __uint_as_float((unsigned)c),
                      __uint_as_float((unsigned)d));
      return true;
    }
    if (ta > e || tb > e || tc > e || td > e) return false;
    if ((++it & 63u) == 0 && now_ns() > deadline) return false;
  }
}
__device__ __forceinline__ bool ll_get1(const u64* src, int e, unsigned long long deadline, float& v) {
  unsigned it = 0;
  for (;;) {
    u64 a;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(a) : "l"(src) : "memory");
    const int ta = (int)(a >> 32);
    if (ta == e) {
      v = __uint_as_float((unsigned)a);
      return true;
    }
    if (ta > e) return false;
    if ((++it & 63u) == 0 && now_ns() > deadline) return false;
  }
}

// Final rows in the output's 16-bit type (owner mode): a pair of values per
// word (packed as the output stores them) and the step in the high half, so
// the hand-back moves half the bytes of fp32 words and the receivers write
// exactly what the owner writes.
template <typename T>
__device__ __forceinline__ void ll_put4h(u64* dst, float4 v, int e) {
  const u64 a = ((u64)(unsigned)e << 32) | Elem<T>::pack2(v.x, v.y);
  const u64 b = ((u64)(unsigned)e << 32) | Elem<T>::pack2(v.z, v.w);
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a), "l"(b) : "memory");
}
template <typename T>
__device__ __forceinline__ float2 unpack_pair(unsigned w) {
  T lo, hi;
  const unsigned short wl = (unsigned short)(w & 0xffffu), wh = (unsigned short)(w >> 16);
  memcpy(&lo, &wl, 2);
  memcpy(&hi, &wh, 2);
  return make_float2(Elem<T>::to_f(lo), Elem<T>::to_f(hi));
}
template <typename T>
__device__ __forceinline__ bool ll_get4h(const u64* src, int e, unsigned long long deadline, float4& v) {
  unsigned it = 0;
  for (;;) {
    u64 a, b;
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(src) : "memory");
    const int ta = (int)(a >> 32), tb = (int)(b >> 32);
    if (ta == e && tb == e) {
      const float2 x = unpack_pair<T>((unsigned)a), y = unpack_pair<T>((unsigned)b);
      v = make_float4(x.x, x.y, y.x, y.y);
      return true;
    }
    if (ta > e || tb > e) return false;
    if ((++it & 63u) == 0 && now_ns() > deadline) return false;
  }
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

template <typename T, int D, int W, bool OWNED>
__global__ void __launch_bounds__(kThreads, blocks_per_sm(W))
    sharded_combine_kernel(const AttnParams p, const PeerBases pb, int rank, const ExLayout L) {
  constexpr int TPR = D / 4;            // threads per row, one float4 of O each
  constexpr int RPB = kThreads / TPR;   // rows per row block
  char* const mine = pb.base[rank];
  // Every launch over this buffer has the same grid and advances each block's
  // own count once, so all blocks agree on the step.
  int* const steps = reinterpret_cast<int*>(mine + L.steps_off);
  const int e = *reinterpret_cast<volatile int*>(steps + blockIdx.x) + 1;
  const int64_t slot_off = (e & 1) * L.slot_bytes;
  const unsigned long long deadline = now_ns() + 2000000000ull;
  const int q = threadIdx.x % TPR;
  const float nan = __int_as_float(0x7fc00000);
  auto part_o = [&](char* base, int src, int64_t row) {
    return reinterpret_cast<u64*>(base + slot_off) + ((int64_t)src * L.rows + row) * D + 4 * q;
  };
  auto part_l = [&](char* base, int src, int64_t row) {
    return reinterpret_cast<u64*>(base + slot_off + L.lse_off) + (int64_t)src * L.rows + row;
  };
  auto fin_o = [&](char* base, int64_t row) {
    return reinterpret_cast<u64*>(base + slot_off + L.fin_off) + row * D + 4 * q;
  };
  auto fin_oh = [&](char* base, int64_t row) {      // 16-bit output: two values per word
    return reinterpret_cast<u64*>(base + slot_off + L.fin_off) + row * (D / 2) + 2 * q;
  };
  auto fin_l = [&](char* base, int64_t row) {
    return reinterpret_cast<u64*>(base + slot_off + L.fin_lse_off) + row;
  };
  // Three phases over this block's row blocks, so the NVLink round trips of
  // its row blocks overlap instead of running one after another:
  //   A  combine this rank's split partials of each row, keep the result in
  //      this rank's own region of its buffer, push it to the peers (push
  //      mode) or to the row block's owner (owner mode);
  //   B  for each row this rank merges (all rows in push mode, its own row
  //      blocks in owner mode): wait for the peers' words, merge in rank
  //      order, store the outputs (owner mode: and push the final rows);
  //   C  owner mode, row blocks of other ranks: wait for the final rows.
  bool all_ok = true;
  auto row_of = [&](int rb) { return (int64_t)rb * RPB + threadIdx.x / TPR; };
  auto owner_of = [&](int rb) { return OWNED ? (int)((int64_t)rb * W / L.nrb) : rank; };
  auto store_row = [&](int64_t row, const float4& o, float lse) {
    const int bh = (int)(row / p.R);
    const int r = (int)(row - (int64_t)bh * p.R);
    const int b = bh / p.Hkv;
    const int hk = bh - b * p.Hkv;
    int m, h;
    row_coords(p, hk, r, m, h);
    store_out_pair<T>(p, b, m, h, 4 * q, o.x, o.y);
    store_out_pair<T>(p, b, m, h, 4 * q + 2, o.z, o.w);
    if (q == 0) store_row_stats<T>(p, b, m, h, lse);
  };
  for (int rb = blockIdx.x; rb < L.nrb; rb += gridDim.x) {           // A
    const int64_t row = row_of(rb);
    if (row >= L.rows) continue;
    const int owner = owner_of(rb);
    const int bh = (int)(row / p.R);
    float4 own;
    float own_l;
    combine_split_row<D>(p, bh, (int)(row - (int64_t)bh * p.R), q, own, own_l);
    ll_put4(part_o(mine, rank, row), own, e);
    if (q == 0) ll_put1(part_l(mine, rank, row), own_l, e);
#pragma unroll
    for (int pr = 0; pr < W; ++pr) {
      if (pr == rank || (OWNED && pr != owner)) continue;
      ll_put4(part_o(pb.base[pr], rank, row), own, e);
      if (q == 0) ll_put1(part_l(pb.base[pr], rank, row), own_l, e);
    }
  }
  for (int rb = blockIdx.x; rb < L.nrb; rb += gridDim.x) {           // B
    const int64_t row = row_of(rb);
    if (row >= L.rows || owner_of(rb) != rank) continue;
    bool ok = true;
    float l[W];
    float4 v[W];
#pragma unroll
    for (int pr = 0; pr < W; ++pr) {
      ok = ll_get4(part_o(mine, pr, row), e, deadline, v[pr]) && ok;   // own words: already there
      ok = ll_get1(part_l(mine, pr, row), e, deadline, l[pr]) && ok;
    }
    float4 o;
    float lse;
    merge_ranks<W>(l, v, o, lse);
    if (!ok) {
      o = make_float4(nan, nan, nan, nan);
      lse = nan;
    }
    if (OWNED) {
      // Hand the final rows to every other rank.
#pragma unroll
      for (int pr = 0; pr < W; ++pr) {
        if (pr == rank) continue;
        if (p.out_f32) ll_put4(fin_o(pb.base[pr], row), o, e);
        else ll_put4h<T>(fin_oh(pb.base[pr], row), o, e);
        if (q == 0) ll_put1(fin_l(pb.base[pr], row), lse, e);
      }
    }
    all_ok = all_ok && ok;
    store_row(row, o, lse);
  }
  if (OWNED) {
    for (int rb = blockIdx.x; rb < L.nrb; rb += gridDim.x) {         // C
      const int64_t row = row_of(rb);
      if (row >= L.rows || owner_of(rb) == rank) continue;
      float4 o;
      float lse;
      bool ok = p.out_f32 ? ll_get4(fin_o(mine, row), e, deadline, o) : ll_get4h<T>(fin_oh(mine, row), e, deadline, o);
      ok = ll_get1(fin_l(mine, row), e, deadline, lse) && ok;
      if (!ok) {
        o = make_float4(nan, nan, nan, nan);
        lse = nan;
      }
      all_ok = all_ok && ok;
      store_row(row, o, lse);
    }
  }
  if (!all_ok && p.err) atomicExch(p.err, 8);
  __syncthreads();   // every thread has read this block's step count
  if (threadIdx.x == 0) steps[blockIdx.x] = e;
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
  // Every block of the grid must be resident at once: at most
  // blocks_per_sm(world) blocks of 128 threads per SM, each looping over row
  // blocks.
  const int cap = blocks_per_sm(world) * kNumSMs;
  const int grid = L.nrb < cap ? L.nrb : cap;
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

int64_t sharded_exchange_bytes(int world, int64_t rows, int D) { return layout(world, rows, D).total; }

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
