// Verify attention, tensor-memory path: tcgen05 MMA with TMEM accumulators,
// TMA page-tile loads, warp-specialised (sm_100a).
//
// A CTA holds 128 query rows of one (batch, KV head) -- tree nodes times the
// query heads of the GQA group -- and streams one split of the keys in
// 128-key tiles.  The row blocks of one KV head (two at 64 nodes x GQA 4) are
// launched as one cluster so they run on one GPC and share the K/V tiles in
// L2.
//
//   warps 0, 10  TMA producers, all 32 lanes: warp 0 loads K, warp 10 loads V,
//             each with its own ring cursor.  A box is one chunk of up to 16
//             tokens read straight from the paged pool through the page table
//             (page ids a tile ahead) into 128-byte-swizzled tiles; the boxes
//             of a tile are spread over the lanes.  "Wide" boxes carry both
//             64-dim halves of a chunk (4 KB at 16 tokens), "narrow" ones one
//             half (2 KB); wide needs a pool whose page index and head index
//             merge into one stride (the reference's [P, Hkv, page, D]).
//             Missing pages are fetched at an out-of-range index, which TMA
//             fills with zeros.
//   warps 11, 1  MMA issuers (one thread each): S = Q K^T (A = Q, B = K from
//             shared memory, fp32 accumulator in TMEM) and O += P V (A = P
//             read from TMEM, B = V from shared memory), each issued as soon
//             as its inputs are ready.  Before the PV of a tile that ends
//             inside a page, the PV issuer zeroes the V rows past the last
//             key (the page's unused slots may hold anything, and 0 * NaN is
//             NaN).
//   warps 2-9 softmax: warps 2-5 take the even tiles, warps 6-9 the odd ones;
//             warp w covers TMEM lane quarter w % 4, and each thread owns one
//             query row and all 128 keys of its tiles.  The running reference
//             max passes from tile to tile through shared memory; it only
//             moves when a tile's max exceeds it by more than 2^8, so O is
//             rescaled rarely.  The bitmask applies on the tail tiles only.
//
// Tensor memory (512 columns): S0 S1 (fp32 scores, 128 columns each), P0 P1
// (16-bit pairs, 64 columns each), O (128 columns).  S(j) reuses its buffer
// once the softmax warps have read S(j-2); P(i) reuses its buffer once
// PV(i-2) has retired, so a softmax warp never waits for the PV of the tile
// it just finished.
//
// Every mbarrier wait is bounded (2 s); on expiry the CTA raises an abort
// flag, records a status word, poisons its rows with NaN, unwinds and frees
// its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <string.h>

#include <type_traits>

#include "attn_epilogue.cuh"
#include "attn_kernels.cuh"
#include "sm100.cuh"

namespace tv {
namespace {

using namespace sm100;

constexpr int BN = 128;               // keys per tile
constexpr int ROWS = 128;             // query rows per CTA
constexpr int HD = 128;               // head_dim
constexpr int SUB = 128 * 128;        // [128 rows][64 dims] swizzled subtile (16 KB)
constexpr int TILE = 2 * SUB;         // 128 rows x 128 dims (32 KB)
constexpr int ST = 3;                 // ring slots of K and of V
constexpr float kRescale = 8.0f;      // log2 units
constexpr int THREADS = 384;          // K producer, PV issuer, 8 softmax warps, V producer, S issuer
constexpr int SBUF = 2;               // S buffers in TMEM (fp32 scores, 128 columns each)
constexpr int PBUF = 2;               // P buffers in TMEM (16-bit pairs, 64 columns each)
constexpr uint32_t TMEM_COLS = 512;   // S0 S1 P0 P1 O
constexpr uint32_t P_COL = SBUF * BN;
constexpr uint32_t O_COL = P_COL + PBUF * (BN / 2);
static_assert(O_COL + 128 == TMEM_COLS, "tensor memory layout");

constexpr int Q_OFF = 0;
constexpr int K_OFF = TILE;
constexpr int V_OFF = K_OFF + ST * TILE;
constexpr int BAR_OFF = V_OFF + ST * TILE;
constexpr int SMEM = BAR_OFF + 3072;  // barriers, row-max exchange
static_assert(SMEM <= 227 * 1024, "shared memory budget");

// Byte offset of row n (a key), 64-dim half h, inside a K or V slot.
//   narrow: [half][128 rows][128 B]                (16 KB per half)
//   wide:   [row / 8][half][row % 8][128 B]        (2 KB per 8-row group)
// Both are 128-byte-swizzle layouts of 1 KB atoms (8 rows x 128 B).
template <bool WIDE>
__host__ __device__ constexpr int row_off(int n, int h) {
  return WIDE ? (n >> 3) * 2048 + h * 1024 + (n & 7) * 128 : h * SUB + n * 128;
}

struct Bars {
  uint64_t k_full[ST];
  uint64_t k_empty[ST];
  uint64_t v_full[ST];
  uint64_t v_empty[ST];
  uint64_t s_full[SBUF];
  uint64_t s_free[SBUF];    // the 4 softmax warps of a tile have read its scores
  uint64_t p_full[PBUF];    // 4 softmax warps arrive
  uint64_t pv_done[PBUF];   // per P buffer: PV of the tile in it retired
  uint64_t o_done;
  uint64_t pair[4];         // per TMEM lane quarter: the two softmax warps meet at the end
  uint32_t tmem;
  int abort;
  // Per row, the reference max (log2 units) after the latest decided tile in
  // the low half and that tile's index + 1 in the high half of one word: a
  // reader polls its row's word until the tile it needs is there.  At the
  // end the same bytes carry the two warps' final references (xm).
  union {
    uint64_t mref[ROWS];
    float xm[2 * ROWS];     // final references and partial sums of the two warps of a row
  };
  float xl[2 * ROWS];
};
static_assert(sizeof(Bars) <= 3072, "barrier block");

__device__ __forceinline__ void raise_abort(Bars* bars, int* err, int code) {
  bars->abort = 1;
  if (err) atomicExch(err, code);
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  return Elem<T>::pack2(lo, hi);
}

// Low / high 32-bit words of a 128-byte-swizzle shared-memory descriptor
// (start address and leading byte offset in the low word; stride byte offset,
// version 1 and the layout type in the high word).
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t desc_hi(uint32_t sbo_bytes) {
  return ((sbo_bytes >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);
}

__device__ __forceinline__ void mma_ss_w(uint32_t d_tmem, uint32_t a_lo, uint32_t a_hi, uint32_t b_lo, uint32_t b_hi,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 ad, bd;\n\t"
      "mov.b64 ad, {%1, %2};\n\t"
      "mov.b64 bd, {%3, %4};\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %5, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(a_hi), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t b_hi,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 bd;\n\t"
      "mov.b64 bd, {%2, %3};\n\t"
      "setp.ne.b32 p, %5, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], bd, %4, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(b_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// TMA tile load, 5-D map (the wide boxes).
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"((uint32_t)__cvta_generic_to_shared(bar))
      : "memory");
}

// Visibility of the 32 keys rel0 .. rel0+31, counted from the start of the
// bitmask-gated tail: keys before the tail are visible, keys at or past the
// tail's end (the sequence end) are not, the rest follow the row's bits.
__device__ __forceinline__ uint32_t keep_bits(const uint64_t* mrow, int rel0, int mlen) {
  if (rel0 <= -32) return ~0u;
  uint32_t k = rel0 >= 0 ? 0u : ((1u << (-rel0)) - 1u);   // keys before the tail
  const int a = rel0 > 0 ? rel0 : 0;
  const int e = rel0 + 32 < mlen ? rel0 + 32 : mlen;
  if (a < e) {
    const int w = a >> 6, sh = a & 63, cnt = e - a;         // cnt <= 32
    uint64_t bits = mrow[w] >> sh;
    if (sh > 32 && ((w + 1) << 6) < mlen) bits |= mrow[w + 1] << (64 - sh);
    const uint32_t got = (uint32_t)bits & (cnt == 32 ? ~0u : ((1u << cnt) - 1u));
    k |= got << (a - rel0);
  }
  return k;
}

// The reference hand-off word of a row: value bits low, tile index + 1 high;
// one aligned 64-bit shared-memory access is single-copy atomic.
__device__ __forceinline__ void ref_put(uint64_t* w, float v, uint32_t tag) {
  const uint64_t x = ((uint64_t)tag << 32) | __float_as_uint(v);
  asm volatile("st.volatile.shared.u64 [%0], %1;" ::"r"((uint32_t)__cvta_generic_to_shared(w)), "l"(x) : "memory");
}
// Polls until the word carries `tag` (bounded like mbar_wait).
__device__ __forceinline__ bool ref_wait(const uint64_t* w, uint32_t tag, volatile int* abort, float& v) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(w);
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    uint64_t x;
    asm volatile("ld.volatile.shared.u64 %0, [%1];" : "=l"(x) : "r"(a) : "memory");
    if ((uint32_t)(x >> 32) == tag) {
      v = __uint_as_float((uint32_t)x);
      return true;
    }
    if ((it & 255u) == 255u) {
      if (*abort) return false;
      if (global_ns() - t0 > 2000000000ull) return false;
    }
  }
}

// Scores of keys the row may not see become -inf in place (their P is then
// exp2(-inf) = 0), so the max and exp passes below have one code path; only
// the tail tiles pay for it.
__device__ __forceinline__ void apply_keep(uint32_t* v, const uint32_t* keep) {
#pragma unroll
  for (int j = 0; j < 64; ++j)
    if (!((keep[j >> 5] >> (j & 31)) & 1u)) v[j] = 0xff800000u;
}

// Maximum over 64 scores: three-input maxima (two scores per instruction)
// over eight independent chains, which keep the dependent path short.
__device__ __forceinline__ float chunk_max(const uint32_t* v) {
  float mx[8];
#pragma unroll
  for (int a = 0; a < 8; ++a) mx[a] = __uint_as_float(v[a]);
#pragma unroll
  for (int j = 8; j < 64; j += 2) mx[(j >> 1) & 7] = max3(mx[(j >> 1) & 7], __uint_as_float(v[j]), __uint_as_float(v[j + 1]));
  return max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
}

// P = exp2(s * sl2 - mu) for 64 scores, packed as 16-bit pairs (key 2k in the
// low half of word k: the layout the PV MMA reads A from); returns sum of P,
// accumulated as packed pairs (one add per two keys).
template <typename T>
__device__ __forceinline__ float chunk_exp(const uint32_t* v, float sl2, float mu, uint32_t* pk) {
  float2 s[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
  for (int j = 0; j < 64; j += 2) {
    // scale and shift two scores with one packed f32x2 FMA
    const float2 x = fma2(make_float2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])), make_float2(sl2, sl2),
                          make_float2(-mu, -mu));
    const float p0 = fast_exp2(x.x);
    const float p1 = fast_exp2(x.y);
    s[(j >> 1) & 1] = add2(s[(j >> 1) & 1], make_float2(p0, p1));
    pk[j >> 1] = pack_pair<T>(p0, p1);
  }
  return (s[0].x + s[1].x) + (s[0].y + s[1].y);
}

template <typename T, bool PAGED, bool WIDE>
__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                   int box, int tok_first) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 128-byte-swizzled TMA tiles need 1 KB alignment; the budget leaves no
  // room to realign, so an unaligned base is reported instead of used.
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0 && p.err) atomicExch(p.err, 7);
    return;
  }
  uint8_t* smem = smem_raw;
  uint8_t* sQ = smem + Q_OFF;
  uint8_t* sK = smem + K_OFF;
  uint8_t* sV = smem + V_OFF;
  Bars* bars = reinterpret_cast<Bars*>(smem + BAR_OFF);
  volatile int* abort = &bars->abort;
  int* err = p.err;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rb = blockIdx.x;
  const int bh = blockIdx.y;
  const int split = blockIdx.z;
  const int b = bh / p.Hkv;
  const int hk = bh - b * p.Hkv;
  const int len = p.num_keys;
  const int tail = len - p.mask_len;
  const int ntiles = (len + BN - 1) / BN;
  const int t0 = split * p.tiles_per_split;
  const int t1 = min(ntiles, t0 + p.tiles_per_split);
  const int NT = t1 > t0 ? t1 - t0 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    for (int s = 0; s < SBUF; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->s_free[s], 4);
      mbar_init(&bars->p_full[s], 4);
    }
    for (int s = 0; s < PBUF; ++s) mbar_init(&bars->pv_done[s], 1);
    mbar_init(&bars->o_done, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&bars->pair[q], 64);
    bars->abort = 0;
    for (int r = 0; r < ROWS; ++r) bars->mref[r] = 0ull;
    mbar_fence_init();
  }
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
    }
    __syncwarp();
    tmem_alloc(&bars->tmem, TMEM_COLS);
    tmem_relinquish();
  }

  // Barriers and the tensor-memory address are visible after this; the
  // producers start their loads at once, while the other ten warps stage the
  // queries (only the S issuer reads them, after the named barrier below).
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  // ---- queries -> shared memory, 128-byte swizzled [d-half][row][64] --------
  if (warp != 0 && warp != 10) {
    constexpr int QT = THREADS - 64;                       // staging threads
    const int lid = threadIdx.x - (warp < 10 ? 32 : 64);
    const T* qb = static_cast<const T*>(p.q);
    for (int idx = lid; idx < ROWS * 16; idx += QT) {
      const int row = idx >> 4;
      const int c = idx & 15;
      const int r = rb * ROWS + row;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.R) {
        int m, h;
        row_coords(p, hk, r, m, h);
        val = *reinterpret_cast<const uint4*>(qb + (int64_t)b * p.q_sb + (int64_t)m * p.q_sm + (int64_t)h * p.q_sh +
                                              c * 8);
      }
      const int dh = c >> 3, cc = c & 7;
      *reinterpret_cast<uint4*>(sQ + dh * SUB + row * 128 + ((cc ^ (row & 7)) << 4)) = val;
    }
    fence_proxy_async();
    asm volatile("bar.sync 1, %0;" ::"n"(QT) : "memory");
  }

  if (warp == 0 || warp == 10) {
    // ---------------------------------------------------------------- producers
    // Warp 0 loads K, warp 10 loads V, each with its own ring cursor.  One
    // thread keeps about one TMA box in flight (a box costs its issuing
    // thread roughly a memory latency), so a tile's boxes are spread over the
    // lanes, and successive tiles rotate to the next lanes: box j of tile i
    // goes to lane (i * n + j) mod 32, letting a warp keep two or more tiles
    // in flight.  Each warp reads the page ids of the next tile's chunks a
    // tile ahead.
    if (NT > 0) {
      const bool is_k = warp == 0;
      const int nch = BN / box;                        // chunks per tile
      const int nb = WIDE ? nch : 2 * nch;             // boxes per tile
      uint64_t* full_ring = is_k ? bars->k_full : bars->v_full;
      uint64_t* empty_ring = is_k ? bars->k_empty : bars->v_empty;
      const CUtensorMap* map = is_k ? &tmk : &tmv;
      uint8_t* base = is_k ? sK : sV;
      // page id of chunk `lane` of tile t (lanes past the tile's chunks: -1)
      auto fetch_page = [&](int t) {
        const int n0 = t * BN + lane * box;
        return (PAGED && lane < nch && n0 < len) ? p.pt[(int64_t)b * p.pt_sb + (n0 >> p.page_shift)] : -1;
      };
      int cur_pg = PAGED ? fetch_page(t0) : -1;
      const uint64_t t_start = global_ns();
      int i = 0;
      bool failed = false;
      while (i < NT) {
        int go = 1;
        if (i >= ST && lane == 0) {
          go = mbar_try_wait(&empty_ring[i % ST], ((i / ST) & 1) ^ 1);
          if (!go) {
            go = mbar_try_wait_hint(&empty_ring[i % ST], ((i / ST) & 1) ^ 1, 20000u);
            if (!go && *abort) go = -1;
            else if (!go && global_ns() - t_start > 2000000000ull) go = -2;
          }
        }
        go = __shfl_sync(0xffffffffu, go, 0);
        if (go < 0) {
          failed = go == -2;
          break;
        }
        if (!go) continue;
        const int s = i % ST;
        if (lane == 0) mbar_arrive_expect_tx(&full_ring[s], TILE);
        const int pg_now = cur_pg;
        if (PAGED && i + 1 < NT) cur_pg = fetch_page(t0 + i + 1);
        __syncwarp();
        // At most 32 boxes per tile (chunks of >= 8 tokens): one per lane.
        const int bx = (lane - ((i * nb) & 31)) & 31;
        const int c = WIDE ? bx : bx >> 1;
        const int half = WIDE ? 0 : bx & 1;
        const int id = __shfl_sync(0xffffffffu, pg_now, c & 31);   // whole warp: page id of chunk c
        if (bx < nb) {
          const int n0 = (t0 + i) * BN + c * box;
          uint8_t* dst = base + s * TILE + row_off<WIDE>(c * box, half);
          if (WIDE) {
            // 5-D map {64 dims, 8 tokens, 2 halves, page / 8, page * Hkv + head}
            const int off = n0 & ((1 << p.page_shift) - 1);
            const int ph = (id >= 0 && id < p.num_pages) ? id * p.Hkv + hk : p.num_pages * p.Hkv;
            tma_load_5d(dst, map, &full_ring[s], 0, 0, 0, off >> 3, ph);
          } else {
            int c1, c2, c3;
            if (PAGED) {
              const int off = n0 & ((1 << p.page_shift) - 1);
              c1 = tok_first ? off : hk;
              c2 = tok_first ? hk : off;
              c3 = (id >= 0 && id < p.num_pages) ? id : p.num_pages;   // missing page / past the end: zeros
            } else {
              c1 = tok_first ? n0 : hk;
              c2 = tok_first ? hk : n0;
              c3 = b;
            }
            tma_load_4d(dst, map, &full_ring[s], half * 64, c1, c2, c3);
          }
        }
        ++i;
      }
      if (lane == 0) {
        if (failed) raise_abort(bars, err, 1);
        if (*abort) {
          // Let this CTA's loads in flight land before shared memory is released.
          volatile int keep_waiting = 0;
          for (int j = i > ST ? i - ST : 0; j < i; ++j)
            mbar_wait(&full_ring[j % ST], (j / ST) & 1, &keep_waiting, 200000000ull);
        }
      }
    }
  } else if (warp == 1 || warp == 11) {
    // ---------------------------------------------------------------- MMA issuers
    // Two threads feed the tensor pipe: warp 11 issues S(j) = Q K^T as soon
    // as K(j) has landed and the softmax warps have read S(j-2) out of its
    // buffer; warp 1 issues O += P(i) V(i) as soon as P(i) and V(i) are
    // ready.  Each keeps the pipe busy while the other waits.
    if (lane == 0 && NT > 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t id_s = idesc_f16(fmt, 128, BN, 0);
      constexpr uint32_t id_pv = idesc_f16(fmt, 128, HD, 1);
      constexpr uint32_t hi_q = desc_hi(1024);                 // Q: 8-row groups 1 KB apart
      constexpr uint32_t hi_kv = desc_hi(WIDE ? 2048 : 1024);  // K / V: 8-row groups
      const uint32_t q_lo = desc_lo(smem_u32(sQ), 16);
      const uint32_t k_lo = desc_lo(smem_u32(sK), 16);
      // V is MN-major: the leading offset steps between the two 64-dim halves
      const uint32_t v_lo = desc_lo(smem_u32(sV), WIDE ? 1024 : SUB);
      bool ok = true;
      if (warp == 11) {
        for (int j = 0; ok && j < NT; ++j) {
          const int sb = j % SBUF, ks = j % ST;
          // buffer sb is free once the softmax warps have read S(j - SBUF)
          if (j >= SBUF && !mbar_wait(&bars->s_free[sb], ((j - SBUF) / SBUF) & 1, abort)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&bars->k_full[ks], (j / ST) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(sb * BN);
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint32_t qo = (uint32_t)(((kk >> 2) * SUB + (kk & 3) * 32) >> 4);
            const uint32_t ko = (uint32_t)((ks * TILE + row_off<WIDE>(0, kk >> 2) + (kk & 3) * 32) >> 4);
            mma_ss_w(d, q_lo + qo, hi_q, k_lo + ko, hi_kv, id_s, kk > 0 ? 1u : 0u);
          }
          tc_commit(&bars->s_full[sb]);
          tc_commit(&bars->k_empty[ks]);
        }
        if (!ok) raise_abort(bars, err, 2);
      } else {
        for (int i = 0; ok && i < NT; ++i) {
          const int pb = i % PBUF, vs = i % ST;
          if (!mbar_wait(&bars->p_full[pb], (i / PBUF) & 1, abort)) {
            ok = false;
            break;
          }
          if (!mbar_wait(&bars->v_full[vs], (i / ST) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (PAGED) {
            // A tile ending inside a chunk: the chunk's rows past the last key
            // came from unused page slots.  Zero them (both halves) before the
            // PV reads V; chunks starting past the end were zero-filled by TMA.
            const int r0 = len - (t0 + i) * BN;
            if (r0 < BN && (r0 % box) != 0) {
              const int r1 = min(BN, (r0 / box + 1) * box);
              uint8_t* slot = sV + vs * TILE;
              for (int n = r0; n < r1; ++n) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  uint4* row = reinterpret_cast<uint4*>(slot + row_off<WIDE>(n, h));
#pragma unroll
                  for (int c = 0; c < 8; ++c) row[c] = make_uint4(0u, 0u, 0u, 0u);
                }
              }
              fence_proxy_async();   // generic writes before the MMA's async-proxy reads
            }
          }
          const uint32_t a = tmem + P_COL + (uint32_t)(pb * (BN / 2));
#pragma unroll
          for (int kb = 0; kb < BN / 16; ++kb) {
            const uint32_t vo = (uint32_t)((vs * TILE + row_off<WIDE>(16 * kb, 0)) >> 4);
            const uint32_t acc = (i > 0 || kb > 0) ? 1u : 0u;
            mma_ts_w(tmem + O_COL, a + kb * 8, v_lo + vo, hi_kv, id_pv, acc);
          }
          tc_commit(&bars->v_empty[vs]);
          tc_commit(&bars->pv_done[pb]);
        }
        if (ok) tc_commit(&bars->o_done);   // tracks every PV; each followed its S
        else raise_abort(bars, err, 2);
      }
    }
  } else if (warp >= 2 && warp < 10) {
    // ---------------------------------------------------------------- softmax
    // Warps 2-5 take the even tiles, warps 6-9 the odd tiles (tile i in S
    // buffer i % 2), so the two warps sharing a scheduler (and its MUFU unit)
    // work on successive tiles at the same time.  Warp w covers TMEM lane
    // quarter w % 4: each thread owns one query row and all 128 keys of its
    // tiles.  The running reference max passes from tile to tile through
    // shared memory (one tagged word per row, polled by the next tile's
    // thread of the same row); it only moves
    // when a tile's max exceeds it by more than 2^8, and then O is rescaled
    // before that tile's PV.  Each warp keeps a partial row sum against the
    // reference it last saw; the two are combined at the end.
    const int q4 = warp & 3;                      // TMEM lane quarter of this warp
    const int par = (warp - 2) >> 2;              // parity of the tiles this warp takes
    const int rr = q4 * 32 + lane;                // row within the CTA
    const int r = rb * ROWS + rr;
    const bool valid = r < p.R;
    const int m = (valid ? r : p.R - 1) / p.G;
    const uint64_t* mrow = p.mask ? p.mask + (int64_t)b * p.mask_sb + (int64_t)m * p.mask_sm : nullptr;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t o_addr = lane_base + O_COL;
    const float sl2 = p.scale_log2;
    const int mlen = p.mask_len;
    uint64_t* ref_word = &bars->mref[rr];
    uint64_t* pair = &bars->pair[q4];             // both warps of the quarter meet once, at the end
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    // A warp whose 32 rows are all padding (the last row block of an
    // M x G that is not a multiple of 128) keeps every wait and arrival of
    // the pipeline, in the same order, but computes nothing: its P lanes
    // hold whatever they held, which only reaches O rows never stored.  Both
    // warps of a lane quarter cover the same rows, so both skip the
    // reference hand-off.
    const bool live = __any_sync(0xffffffffu, valid);
    for (int i = par; i < NT && !live; i += 2) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[i % SBUF], (i / SBUF) & 1, abort))) {
        raise_abort(bars, err, 3);
        ok = false;
        break;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_free[i % SBUF]);
      if (i >= PBUF && !__all_sync(0xffffffffu, mbar_wait(&bars->pv_done[i % PBUF], ((i - PBUF) / PBUF) & 1, abort))) {
        raise_abort(bars, err, 7);
        ok = false;
        break;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[i % PBUF]);
    }
    for (int i = par; i < NT && live; i += 2) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[i % SBUF], (i / SBUF) & 1, abort))) {
        raise_abort(bars, err, 3);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = lane_base + (uint32_t)((i % SBUF) * BN);
      const int n0 = (t0 + i) * BN;
      // Tiles wholly inside the prefix take the unmasked path; the bitmask is
      // applied only where the tail begins, and not on tiles whose mask words
      // are all ones in every row (the optional word summary).
      bool edge = (n0 + BN > len) || (n0 + BN > tail);
      if (edge && p.mfull && n0 + BN <= len) {
        const int a0 = n0 > tail ? n0 - tail : 0, e0 = n0 + BN - tail;   // gated keys [a0, e0), e0 <= mlen
        bool full = true;
        for (int w = a0 >> 6; w <= (e0 - 1) >> 6; ++w) full = full && p.mfull[(int64_t)b * p.mfull_sb + w] != 0;
        edge = !full;
      }
      uint32_t keep[4] = {~0u, ~0u, ~0u, ~0u};
      if (edge) {
#pragma unroll
        for (int c = 0; c < 4; ++c) keep[c] = keep_bits(mrow, n0 + 32 * c - tail, mlen);
      }
      // Two passes of 64 columns (three warps share a scheduler's registers,
      // so a thread cannot hold all 128 scores): the row max, then P.
      uint32_t v[64];
      tmem_ld32(s_addr, v);
      tmem_ld32(s_addr + 32, v + 32);
      tmem_wait_ld();
      if (edge) apply_keep(v, keep);
      float mx = chunk_max(v);
      tmem_ld32(s_addr + 64, v);
      tmem_ld32(s_addr + 96, v + 32);
      tmem_wait_ld();
      if (edge) apply_keep(v, keep + 2);
      mx = fmaxf(mx, chunk_max(v));
      // pass 2's first scores are loaded now; the latency hides behind the
      // hand-off below
      tmem_ld32(s_addr, v);
      tmem_ld32(s_addr + 32, v + 32);
      // Reference after tile i-1 (published by the other warp of the quarter).
      float mprev = -INFINITY;
      if (i > 0) {
        if (!__all_sync(0xffffffffu, ref_wait(ref_word, (uint32_t)i, abort, mprev))) {
          raise_abort(bars, err, 6);
          ok = false;
          break;
        }
      }
      if (mprev > m_run) {          // the reference only grows
        l_run *= fast_exp2(m_run - mprev);
        m_run = mprev;
      }
      const float mt = mx * sl2;
      float alpha = 1.f;
      const bool bump = mt > m_run + kRescale;
      if (bump) {
        alpha = fast_exp2(m_run - mt);
        m_run = mt;
      }
      ref_put(ref_word, m_run, (uint32_t)i + 1u);   // reference for tile i+1
      const bool need_o = bump && i > 0;
      if (__any_sync(0xffffffffu, need_o)) {
        // O holds tiles up to i-1 scaled to mprev; PV(i-1) must retire first.
        // PV(i-2) is waited for on this warp's own P-buffer barrier (exact:
        // its tile i-4 phase was observed before P(i-2) was written); PVs
        // retire in order, so the other buffer's barrier then stands at tile
        // i-1 and that wait is exact too.  PV(i) waits for p_full below.
        bool got = true;
        if (i >= 2) got = mbar_wait(&bars->pv_done[i % PBUF], ((i - 2) / PBUF) & 1, abort);
        if (got) got = mbar_wait(&bars->pv_done[(i - 1) % PBUF], ((i - 1) / PBUF) & 1, abort);
        if (!__all_sync(0xffffffffu, got)) {
          raise_abort(bars, err, 4);
          ok = false;
          break;
        }
        tc_fence_after();
        const float a = need_o ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t ov[32];
          tmem_ld32(o_addr + 32 * c, ov);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = __float_as_uint(__uint_as_float(ov[j]) * a);
          tmem_st32(o_addr + 32 * c, ov);
        }
      }
      l_run *= alpha;
      const float mu = m_run == -INFINITY ? 0.f : m_run;
      // P: keys 0-63 into P-buffer columns 0-31, keys 64-127 into 32-63.
      uint32_t pk[32];
      tmem_wait_ld();
      if (edge) apply_keep(v, keep);
      l_run += chunk_exp<T>(v, sl2, mu, pk);
      tmem_ld32(s_addr + 64, v);
      tmem_ld32(s_addr + 96, v + 32);
      tmem_wait_ld();
      // All of S(i) is in registers: its buffer can take S(i + SBUF).
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s_free[i % SBUF]);
      // P buffer i % PBUF held P(i - 2), this warp's own previous tile, whose
      // PV was issued right after it, so this wait rarely blocks.  Its phase
      // for tile i - 4 completed before this warp wrote P(i - 2), so the
      // parity wait is exact.
      if (i >= PBUF && !__all_sync(0xffffffffu, mbar_wait(&bars->pv_done[i % PBUF], ((i - PBUF) / PBUF) & 1, abort))) {
        raise_abort(bars, err, 7);
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t p_addr = lane_base + P_COL + (uint32_t)((i % PBUF) * (BN / 2));
      tmem_st32(p_addr, pk);
      if (edge) apply_keep(v, keep + 2);
      l_run += chunk_exp<T>(v, sl2, mu, pk);
      tmem_st32(p_addr + 32, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[i % PBUF]);
    }
    // ---- epilogue -------------------------------------------------------------
    if (ok && NT > 0 && !__all_sync(0xffffffffu, mbar_wait(&bars->o_done, 0, abort))) {
      raise_abort(bars, err, 5);
      ok = false;
    }
    tc_fence_after();
    // Both warps' partial sums, brought to the final reference (the larger of
    // the two, as the reference only grows); the pair barrier's only phase.
    {
      bars->xm[par * ROWS + rr] = m_run;
      bars->xl[par * ROWS + rr] = l_run;
      mbar_arrive(pair);
      if (ok && !__all_sync(0xffffffffu, mbar_wait(pair, 0, abort))) {
        raise_abort(bars, err, 6);
        ok = false;
      }
      const float m2 = bars->xm[(par ^ 1) * ROWS + rr];
      const float l2 = bars->xl[(par ^ 1) * ROWS + rr];
      const float mf = fmaxf(m_run, m2);
      if (mf != -INFINITY) {
        l_run = (m_run == mf ? l_run : l_run * fast_exp2(m_run - mf)) + (m2 == mf ? l2 : l2 * fast_exp2(m2 - mf));
        m_run = mf;
      }
    }
    ok = ok && !*abort;
    const bool have = ok && NT > 0 && l_run > 0.f;
    // A CTA that gave up on a wait poisons its rows so the failure cannot pass
    // for a result; the status word says why.
    const float poison = ok ? 0.f : __int_as_float(0x7fc00000);
    const float inv = have ? 1.f / l_run : 0.f;
    const float lse = have ? (m_run + __log2f(l_run)) * kLn2 : (ok ? -INFINITY : poison);
    const int ch = par;                           // this warp writes head-dim columns ch*64 .. +63
    int mm = 0, hh = 0;
    if (valid) row_coords(p, hk, r, mm, hh);
    float* prow = valid && p.part_o ? part_o_row(p, split, bh, r, HD) : nullptr;
    const int d0 = ch * (HD / 2);
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      uint32_t v[32];
      if (NT > 0) {   // warp-uniform: tcgen05.ld is a warp-collective instruction
        tmem_ld32(o_addr + d0 + 32 * c, v);
        tmem_wait_ld();
      }
      if (valid) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float o0 = have ? __uint_as_float(v[j]) * inv : poison;
          const float o1 = have ? __uint_as_float(v[j + 1]) * inv : poison;
          const float o2 = have ? __uint_as_float(v[j + 2]) * inv : poison;
          const float o3 = have ? __uint_as_float(v[j + 3]) * inv : poison;
          if (prow) {
            *reinterpret_cast<float4*>(prow + d0 + 32 * c + j) = make_float4(o0, o1, o2, o3);
          } else {
            store_out_pair<T>(p, b, mm, hh, d0 + 32 * c + j, o0, o1);
            store_out_pair<T>(p, b, mm, hh, d0 + 32 * c + j + 2, o2, o3);
          }
        }
      }
    }
    if (valid && ch == 0) {
      if (prow) *part_lse_row(p, split, bh, r) = lse;
      else store_row_stats<T>(p, b, mm, hh, lse);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---- host side ------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

CUtensorMapDataType map_type(int dtype) {
  return dtype == TV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

// 4-D map over a KV tensor: head_dim, then tokens and heads in order of
// increasing stride, then the batch / page index.  Box = 64 x box_tok rows
// (one 64-dim half of a chunk).
bool make_map(CUtensorMap* map, int dtype, const void* base, uint64_t ntok, uint64_t nhead, uint64_t nouter,
              int64_t s_tok, int64_t s_head, int64_t s_outer, uint32_t box_tok, bool tok_first) {
  auto enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[4], strides[3];
  cuuint32_t box[4], estr[4] = {1, 1, 1, 1};
  dims[0] = HD;
  box[0] = 64;
  if (tok_first) {
    dims[1] = ntok; dims[2] = nhead; strides[0] = s_tok * 2; strides[1] = s_head * 2;
    box[1] = box_tok; box[2] = 1;
  } else {
    dims[1] = nhead; dims[2] = ntok; strides[0] = s_head * 2; strides[1] = s_tok * 2;
    box[1] = 1; box[2] = box_tok;
  }
  dims[3] = nouter;
  strides[2] = (s_outer > 0 ? s_outer : (int64_t)dims[1] * dims[2] * HD) * 2;
  box[3] = 1;
  const CUresult r = enc(map, map_type(dtype), 4, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 5-D map of a paged pool whose page and head indices merge (page stride =
// heads x head stride): {64 dims, 8 tokens, 2 halves (128 B apart), page / 8
// token groups, page * heads + head}.  One box = box_tok tokens of one head,
// both halves, landing as [token / 8][half][token % 8][128 B].
bool make_wide_map(CUtensorMap* map, int dtype, const void* base, uint64_t page, uint64_t nhead, uint64_t npages,
                   int64_t s_tok, int64_t s_head, uint32_t box_tok) {
  auto enc = encoder();
  if (!enc) return false;
  cuuint64_t dims[5] = {64, 8, 2, page / 8, npages * nhead};
  cuuint64_t strides[4] = {(cuuint64_t)s_tok * 2, 128, (cuuint64_t)s_tok * 16, (cuuint64_t)s_head * 2};
  cuuint32_t box[5] = {64, 8, 2, box_tok / 8, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  const CUresult r = enc(map, map_type(dtype), 5, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, bool PAGED, bool WIDE>
int launch_t(const AttnParams& p, const CUtensorMap& mk, const CUtensorMap& mv, int box, int tok_first,
             cudaStream_t st) {
  auto kern = attn_tc_kernel<T, PAGED, WIDE>;
  const int rc_smem = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), SMEM);
  if (rc_smem != TV_OK) return rc_smem;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tc_row_blocks(p.R), p.B * p.Hkv, p.splits);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  // The row blocks of a KV head read the same K/V tiles: launched as a
  // cluster they run on one GPC, so on one die, and the second read of every
  // tile stays near (measured ~4 % faster at config 2; clusters over several
  // KV heads leave too few free GPC slots for one wave and halve the speed).
  attr[0].val.clusterDim.x = (tc_row_blocks(p.R) % 2 == 0) ? 2 : 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, mk, mv, box, tok_first);
  if (e != cudaSuccess) return record_cuda_error(e);
  return check_launch();
}

}  // namespace

bool tc_supported(int dtype, int D, int R, bool paged, int page_shift) {
  if (D != HD || R < 64) return false;
  if (dtype != TV_BF16 && dtype != TV_F16) return false;
  if (paged && page_shift < 3) return false;    // boxes of at least 8 rows
  return encoder() != nullptr;
}
int tc_tile_keys() { return BN; }
int tc_rows_per_cta() { return ROWS; }
int tc_row_blocks(int R) { return (R + ROWS - 1) / ROWS; }

// The K and V tensor maps of a request; `wide` tells which box layout they
// describe.  kernel bit 7 (128) forces the narrow (half-head) boxes on a
// paged pool.
int tc_maps(const AttnParams& p, int dtype, int kernel_bits, CUtensorMap* mk, CUtensorMap* mv, int* box_out,
            bool* wide) {
  const bool paged = p.pt != nullptr;
  // 16-token boxes (or whole pages of 8): enough boxes per tile to keep
  // every producer lane's load in flight.
  const int box = paged && (1 << p.page_shift) < 16 ? (1 << p.page_shift) : 16;
  const bool tok_first = p.k_sn <= p.k_sh;
  if ((p.v_sn <= p.v_sh) != tok_first) return TV_ERR_UNSUPPORTED;
  *box_out = box;
  *wide = false;
  if (paged) {
    const uint64_t page = 1u << p.page_shift;
    const bool wide_ok = !(kernel_bits & 128) && tok_first && p.k_sb == (int64_t)p.Hkv * p.k_sh &&
                         p.v_sb == (int64_t)p.Hkv * p.v_sh && (int64_t)p.num_pages * p.Hkv < (1ll << 31) - p.Hkv;
    if (wide_ok && make_wide_map(mk, dtype, p.k, page, p.Hkv, p.num_pages, p.k_sn, p.k_sh, box) &&
        make_wide_map(mv, dtype, p.v, page, p.Hkv, p.num_pages, p.v_sn, p.v_sh, box)) {
      *wide = true;
      return TV_OK;
    }
    if (!make_map(mk, dtype, p.k, page, p.Hkv, p.num_pages, p.k_sn, p.k_sh, p.k_sb, box, tok_first) ||
        !make_map(mv, dtype, p.v, page, p.Hkv, p.num_pages, p.v_sn, p.v_sh, p.v_sb, box, tok_first))
      return TV_ERR_UNSUPPORTED;
    return TV_OK;
  }
  if (!make_map(mk, dtype, p.k, p.num_keys, p.Hkv, p.B, p.k_sn, p.k_sh, p.k_sb, box, tok_first) ||
      !make_map(mv, dtype, p.v, p.num_keys, p.Hkv, p.B, p.v_sn, p.v_sh, p.v_sb, box, tok_first))
    return TV_ERR_UNSUPPORTED;
  return TV_OK;
}

// The last few requests' tensor maps, per host thread: a decode loop calls
// with the same caches (one per layer) every step, and encoding a map costs
// microseconds of host time.  The key is everything a map is built from.
struct MapKey {
  const void* k;
  const void* v;
  int64_t k_sb, k_sn, k_sh, v_sb, v_sn, v_sh;
  int64_t n1, n2;           // paged: page shift, pages; contiguous: keys, batch
  int dtype, hkv, paged, narrow;
};
struct MapEntry {
  MapKey key;
  CUtensorMap mk, mv;
  int box;
  bool wide;
  bool used;
};
constexpr int kMapCache = 64;

int tc_maps_cached(const AttnParams& p, int dtype, int kernel_bits, CUtensorMap* mk, CUtensorMap* mv, int* box,
                   bool* wide) {
  static thread_local MapEntry cache[kMapCache];
  static thread_local int next = 0;
  MapKey key;
  memset(&key, 0, sizeof(key));
  key.k = p.k;
  key.v = p.v;
  key.k_sb = p.k_sb; key.k_sn = p.k_sn; key.k_sh = p.k_sh;
  key.v_sb = p.v_sb; key.v_sn = p.v_sn; key.v_sh = p.v_sh;
  key.paged = p.pt != nullptr;
  key.n1 = key.paged ? p.page_shift : p.num_keys;
  key.n2 = key.paged ? p.num_pages : p.B;
  key.dtype = dtype;
  key.hkv = p.Hkv;
  key.narrow = (kernel_bits & 128) ? 1 : 0;
  for (int i = 0; i < kMapCache; ++i) {
    if (cache[i].used && memcmp(&cache[i].key, &key, sizeof(key)) == 0) {
      *mk = cache[i].mk;
      *mv = cache[i].mv;
      *box = cache[i].box;
      *wide = cache[i].wide;
      return TV_OK;
    }
  }
  const int rc = tc_maps(p, dtype, kernel_bits, mk, mv, box, wide);
  if (rc != TV_OK) return rc;
  MapEntry& e = cache[next];
  next = (next + 1) % kMapCache;
  e.key = key;
  e.mk = *mk;
  e.mv = *mv;
  e.box = *box;
  e.wide = *wide;
  e.used = true;
  return TV_OK;
}

int launch_attn_tc(const AttnParams& p, int dtype, int D, int kernel_bits, cudaStream_t st) {
  if (D != HD) return TV_ERR_UNSUPPORTED;
  CUtensorMap mk, mv;
  int box = 16;
  bool wide = false;
  const int rc = tc_maps_cached(p, dtype, kernel_bits, &mk, &mv, &box, &wide);
  if (rc != TV_OK) return rc;
  const int tf = p.k_sn <= p.k_sh ? 1 : 0;
  if (p.pt) {
    if (wide)
      return dtype == TV_BF16 ? launch_t<__nv_bfloat16, true, true>(p, mk, mv, box, tf, st)
                              : launch_t<__half, true, true>(p, mk, mv, box, tf, st);
    return dtype == TV_BF16 ? launch_t<__nv_bfloat16, true, false>(p, mk, mv, box, tf, st)
                            : launch_t<__half, true, false>(p, mk, mv, box, tf, st);
  }
  return dtype == TV_BF16 ? launch_t<__nv_bfloat16, false, false>(p, mk, mv, box, tf, st)
                          : launch_t<__half, false, false>(p, mk, mv, box, tf, st);
}

int attn_tc_wide(const AttnParams& p, int dtype, int kernel_bits) {
  CUtensorMap mk, mv;
  int box = 16;
  bool wide = false;
  return tc_maps(p, dtype, kernel_bits, &mk, &mv, &box, &wide) == TV_OK && wide ? 1 : 0;
}

}  // namespace tv
