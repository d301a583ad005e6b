// Verify attention, tensor-memory path: tcgen05 MMA with TMEM accumulators,
// TMA page-tile loads, warp-specialised (sm_100a).
//
// One CTA holds up to 256 query rows of one (batch, KV head) -- every tree
// node times every query head of the GQA group -- so each 128-key K/V tile
// is read from HBM once for all of them, and streams one split of the keys.
//
//   warp 0        TMA producer: for each 128-key tile, one box per page (per
//                 64-wide half of head_dim) straight from the paged pool via
//                 the page table (or one box per half for a contiguous
//                 cache) into a 2-stage ring of 128-byte-swizzled tiles.
//                 Missing pages are fetched at an out-of-range page index,
//                 which TMA fills with zeros.
//   warp 1        MMA issuer (one thread): S_h = Q_h K^T (A = Q, B = K, both
//                 from shared memory, fp32 accumulators in TMEM), then
//                 O_h += P_h V (A = P read from TMEM, B = V from shared
//                 memory).  tcgen05.commit arrives on mbarriers when groups
//                 of MMAs retire.
//   warps 2..     softmax, one warpgroup per 128-row half h: each thread owns
//                 one query row (one TMEM lane), reads its 128 scores with
//                 tcgen05.ld, applies the tree bitmask, updates the running
//                 max / sum, and writes P (bf16 pairs) back over the scores.
//                 The running max is only moved when it grows by more than
//                 2^8, so O (in TMEM) is rescaled rarely; the final division
//                 uses the same reference point, so the result is exact.
//
// TMEM columns: S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512)
// (one half: S_0 [0,128) O_0 [128,256)).  The two halves ping-pong: while a
// warpgroup works on S_0 the tensor core computes S_1, and so on.
//
// Every mbarrier wait is bounded (2 s); on expiry the CTA raises an abort
// flag, records an error word, unwinds and frees its tensor memory.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <type_traits>

#include "attn_epilogue.cuh"
#include "attn_kernels.cuh"
#include "sm100.cuh"

namespace tv {
namespace {

using namespace sm100;

constexpr int BN = 128;               // keys per tile
constexpr int HALF = 128;             // query rows per MMA (M)
constexpr int HD = 128;               // head_dim
constexpr int STAGES = 2;
constexpr int SUB = 128 * 128;        // one [128 rows][64 elems] swizzled subtile (16 KB)
constexpr int TILE = 2 * SUB;         // 128 rows x 128 dims (32 KB)
constexpr float kRescale = 8.0f;      // log2 units

template <int NH>
struct Layout {
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = NH * TILE;
  static constexpr int V_OFF = K_OFF + STAGES * TILE;
  static constexpr int BAR_OFF = V_OFF + STAGES * TILE;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;   // barriers + alignment slack
  static constexpr int THREADS = 64 + NH * 128;
  static constexpr uint32_t TMEM_COLS = NH == 2 ? 512 : 256;
};

struct Bars {
  uint64_t kv_full[STAGES];
  uint64_t kv_empty[STAGES];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint32_t tmem;
  int abort;
};

__device__ __forceinline__ void raise_abort(Bars* bars, int* err, int code) {
  bars->abort = 1;
  if (err) atomicExch(err, code);
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float lo, float hi) {
  return Elem<T>::pack2(lo, hi);
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

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

template <typename T, int NH, bool PAGED>
__global__ void __launch_bounds__(Layout<NH>::THREADS, 1)
    attn_tc_kernel(const AttnParams p, const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                   int box_tok, int tok_first) {
  using L = Layout<NH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::Q_OFF;
  uint8_t* sK = smem + L::K_OFF;
  uint8_t* sV = smem + L::V_OFF;
  Bars* bars = reinterpret_cast<Bars*>(smem + L::BAR_OFF);
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
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&bars->kv_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&bars->s_full[h], 1);
      mbar_init(&bars->p_full[h], 4);
    }
    mbar_init(&bars->o_done, 1);
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmk);
      prefetch_tmap(&tmv);
    }
    __syncwarp();
    tmem_alloc(&bars->tmem, L::TMEM_COLS);
    tmem_relinquish();
  }

  // ---- queries -> shared memory, 128-byte swizzled [half][d-half][row][64] --------
  {
    const T* qb = static_cast<const T*>(p.q);
    for (int idx = threadIdx.x; idx < NH * HALF * 16; idx += L::THREADS) {
      const int row = idx >> 4;
      const int c = idx & 15;
      const int r = rb * NH * HALF + row;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < p.R) {
        int m, h;
        row_coords(p, hk, r, m, h);
        val = *reinterpret_cast<const uint4*>(qb + (int64_t)b * p.q_sb + (int64_t)m * p.q_sm + (int64_t)h * p.q_sh +
                                              c * 8);
      }
      const int half = row >> 7, rr = row & 127, dh = c >> 3, cc = c & 7;
      *reinterpret_cast<uint4*>(sQ + half * TILE + dh * SUB + rr * 128 + ((cc ^ (rr & 7)) << 4)) = val;
    }
  }
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    if (lane == 0 && NT > 0) {
      int issued = 0;
      for (int i = 0; i < NT; ++i) {
        const int s = i % STAGES;
        if (i >= STAGES && !mbar_wait(&bars->kv_empty[s], ((i / STAGES) & 1) ^ 1, abort)) {
          raise_abort(bars, err, 1);
          break;
        }
        if (*abort) break;
        mbar_arrive_expect_tx(&bars->kv_full[s], 2 * TILE);
        const int t = t0 + i;
        uint8_t* dk = sK + s * TILE;
        uint8_t* dv = sV + s * TILE;
        if (PAGED) {
          const int nbox = BN / box_tok;
          for (int j = 0; j < nbox; ++j) {
            const int n0 = t * BN + j * box_tok;
            int page = p.num_pages;  // out of range: TMA fills zeros
            if (n0 < len) {
              const int pg = p.pt[(int64_t)b * p.pt_sb + (n0 >> p.page_shift)];
              if (pg >= 0 && pg < p.num_pages) page = pg;
            }
            const int off = n0 & ((1 << p.page_shift) - 1);
            const int c1 = tok_first ? off : hk, c2 = tok_first ? hk : off;
#pragma unroll
            for (int dh = 0; dh < 2; ++dh) {
              tma_load_4d(dk + dh * SUB + j * box_tok * 128, &tmk, &bars->kv_full[s], dh * 64, c1, c2, page);
              tma_load_4d(dv + dh * SUB + j * box_tok * 128, &tmv, &bars->kv_full[s], dh * 64, c1, c2, page);
            }
          }
        } else {
          const int n0 = t * BN;
          const int c1 = tok_first ? n0 : hk, c2 = tok_first ? hk : n0;
#pragma unroll
          for (int dh = 0; dh < 2; ++dh) {
            tma_load_4d(dk + dh * SUB, &tmk, &bars->kv_full[s], dh * 64, c1, c2, b);
            tma_load_4d(dv + dh * SUB, &tmv, &bars->kv_full[s], dh * 64, c1, c2, b);
          }
        }
        issued = i + 1;
      }
      if (*abort) {
        // Let this CTA's loads in flight land before shared memory is released.
        volatile int keep_waiting = 0;
        for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i)
          mbar_wait(&bars->kv_full[i % STAGES], (i / STAGES) & 1, &keep_waiting, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0 && NT > 0) {
      const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t id_s = idesc_f16(fmt, HALF, BN, 0);
      const uint32_t id_pv = idesc_f16(fmt, HALF, HD, 1);
      const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
      bool ok = mbar_wait(&bars->kv_full[0], 0, abort);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < NH; ++h) {
#pragma unroll 1
          for (int kk = 0; kk < HD / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sQa + h * TILE + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
            const uint64_t bd = smem_desc_sw128(sKa + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
            mma_ss(tmem + h * 128, ad, bd, id_s, kk > 0);
          }
          tc_commit(&bars->s_full[h]);
        }
      }
      for (int i = 0; ok && i < NT; ++i) {
        const int s = i % STAGES;
        for (int h = 0; h < NH; ++h) {
          if (!mbar_wait(&bars->p_full[h], i & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int kb = 0; kb < BN / 16; ++kb) {
            const uint64_t bd = smem_desc_sw128(sVa + s * TILE + kb * 2048, SUB, 1024);
            mma_ts(tmem + NH * 128 + h * 128, tmem + h * 128 + kb * 8, bd, id_pv, (i > 0 || kb > 0) ? 1u : 0u);
          }
          if (h == NH - 1) tc_commit(&bars->kv_empty[s]);
          if (i + 1 < NT) {
            const int s2 = (i + 1) % STAGES;
            if (h == 0) {
              if (!mbar_wait(&bars->kv_full[s2], ((i + 1) / STAGES) & 1, abort)) {
                ok = false;
                break;
              }
              tc_fence_after();
            }
#pragma unroll 1
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint64_t ad = smem_desc_sw128(sQa + h * TILE + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
              const uint64_t bd = smem_desc_sw128(sKa + s2 * TILE + (kk >> 2) * SUB + (kk & 3) * 32, 16, 1024);
              mma_ss(tmem + h * 128, ad, bd, id_s, kk > 0);
            }
            tc_commit(&bars->s_full[h]);
          }
        }
      }
      tc_commit(&bars->o_done);
      if (!ok) raise_abort(bars, err, 2);
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int h = (warp - 2) >> 2;
    const int q4 = warp & 3;                      // TMEM lane quarter of this warp
    const int rr = q4 * 32 + lane;                // row within the half
    const int r = rb * NH * HALF + h * HALF + rr;
    const bool valid = r < p.R;
    const int m = (valid ? r : p.R - 1) / p.G;
    const uint64_t* mrow = p.mask ? p.mask + (int64_t)b * p.mask_sb + (int64_t)m * p.mask_sm : nullptr;
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    const uint32_t s_addr = lane_base + h * 128;
    const uint32_t o_addr = lane_base + NH * 128 + h * 128;
    const float sl2 = p.scale_log2;
    const int mlen = p.mask_len;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    uint32_t v[32];
    for (int i = 0; i < NT; ++i) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->s_full[h], i & 1, abort))) {
        raise_abort(bars, err, 3);
        ok = false;
        break;
      }
      tc_fence_after();
      const int n0 = (t0 + i) * BN;
      const bool edge = (n0 + BN > len) || (n0 + BN > tail);
      // Pass 1: row maximum over the tile (masked keys excluded).
      uint32_t keep[4] = {~0u, ~0u, ~0u, ~0u};
      if (edge) {
#pragma unroll
        for (int c = 0; c < 4; ++c) keep[c] = keep_bits(mrow, n0 + 32 * c - tail, mlen);
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(s_addr + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if ((keep[c] >> j) & 1u) mx = fmaxf(mx, __uint_as_float(v[j]));
      }
      const float mt = mx * sl2;
      float alpha = 1.f;
      const bool bump = mt > m_run + kRescale;
      if (bump) {
        alpha = fast_exp2(m_run - mt);
        m_run = mt;
      }
      const bool need_o = bump && l_run > 0.f;
      if (__any_sync(0xffffffffu, need_o)) {
        // O_h holds earlier tiles; the tensor pipe finished it before this
        // tile's S_h (same issuing thread, in order), and the next PV into
        // O_h waits for p_full below.
        const float a = need_o ? alpha : 1.f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(o_addr + 32 * c, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) * a);
          tmem_st32(o_addr + 32 * c, v);
        }
      }
      l_run *= alpha;
      const float mu = m_run == -INFINITY ? 0.f : m_run;
      // Pass 2: P = exp2(s * scale * log2e - m) as bf16 pairs over the scores.
      float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        tmem_ld32(s_addr + 32 * c, v);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float p0 = ((keep[c] >> j) & 1u) ? fast_exp2(fmaf(__uint_as_float(v[j]), sl2, -mu)) : 0.f;
          const float p1 = ((keep[c] >> (j + 1)) & 1u) ? fast_exp2(fmaf(__uint_as_float(v[j + 1]), sl2, -mu)) : 0.f;
          sum0 += p0;
          sum1 += p1;
          pk[j >> 1] = pack_pair<T>(p0, p1);
        }
        tmem_st16(s_addr + 16 * c, pk);
      }
      l_run += sum0 + sum1;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->p_full[h]);
    }
    // ---- epilogue -------------------------------------------------------------
    if (ok && NT > 0 && !__all_sync(0xffffffffu, mbar_wait(&bars->o_done, 0, abort))) {
      raise_abort(bars, err, 4);
      ok = false;
    }
    tc_fence_after();
    const bool have = ok && NT > 0 && l_run > 0.f;
    // A CTA that gave up on a wait poisons its rows so the failure cannot pass
    // for a result; the status word says why.
    const float poison = ok ? 0.f : __int_as_float(0x7fc00000);
    const float inv = have ? 1.f / l_run : 0.f;
    const float lse = have ? (m_run + __log2f(l_run)) * kLn2 : (ok ? -INFINITY : poison);
    int mm = 0, hh = 0;
    if (valid) row_coords(p, hk, r, mm, hh);
    float* prow = valid && p.splits > 1 ? part_o_row(p, split, bh, r, HD) : nullptr;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (NT > 0) {   // warp-uniform: tcgen05.ld is a warp-collective instruction
        tmem_ld32(o_addr + 32 * c, v);
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
            *reinterpret_cast<float4*>(prow + 32 * c + j) = make_float4(o0, o1, o2, o3);
          } else {
            store_out_pair<T>(p, b, mm, hh, 32 * c + j, o0, o1);
            store_out_pair<T>(p, b, mm, hh, 32 * c + j + 2, o2, o3);
          }
        }
      }
    }
    if (valid) {
      if (prow) *part_lse_row(p, split, bh, r) = lse;
      else store_row_stats<T>(p, b, mm, hh, lse);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
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

// 4-D map over a KV tensor: head_dim, then tokens and heads in order of
// increasing stride, then the batch / page index.  Box = 64 x box_tok rows.
bool make_map(CUtensorMap* map, int dtype, const void* base, uint64_t ntok, uint64_t nhead, uint64_t nouter,
              int64_t s_tok, int64_t s_head, int64_t s_outer, uint32_t box_tok, bool tok_first) {
  auto enc = encoder();
  if (!enc) return false;
  const CUtensorMapDataType dt = dtype == TV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
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
  const CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename T, int NH, bool PAGED>
int launch_t(const AttnParams& p, const CUtensorMap& mk, const CUtensorMap& mv, int box_tok, int tok_first,
             cudaStream_t st) {
  using L = Layout<NH>;
  auto kern = attn_tc_kernel<T, NH, PAGED>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
  if (e != cudaSuccess) return record_cuda_error(e);
  dim3 grid((p.R + NH * HALF - 1) / (NH * HALF), p.B * p.Hkv, p.splits);
  kern<<<grid, L::THREADS, L::SMEM, st>>>(p, mk, mv, box_tok, tok_first);
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
int tc_rows_per_cta() { return 2 * HALF; }

int launch_attn_tc(const AttnParams& p, int dtype, int D, cudaStream_t st) {
  if (D != HD) return TV_ERR_UNSUPPORTED;
  const bool paged = p.pt != nullptr;
  const int box_tok = paged ? ((1 << p.page_shift) < BN ? (1 << p.page_shift) : BN) : BN;
  const bool tok_first = p.k_sn <= p.k_sh;
  if ((p.v_sn <= p.v_sh) != tok_first) return TV_ERR_UNSUPPORTED;
  CUtensorMap mk, mv;
  bool ok;
  if (paged) {
    ok = make_map(&mk, dtype, p.k, 1u << p.page_shift, p.Hkv, p.num_pages, p.k_sn, p.k_sh, p.k_sb, box_tok, tok_first) &&
         make_map(&mv, dtype, p.v, 1u << p.page_shift, p.Hkv, p.num_pages, p.v_sn, p.v_sh, p.v_sb, box_tok, tok_first);
  } else {
    ok = make_map(&mk, dtype, p.k, p.num_keys, p.Hkv, p.B, p.k_sn, p.k_sh, p.k_sb, box_tok, tok_first) &&
         make_map(&mv, dtype, p.v, p.num_keys, p.Hkv, p.B, p.v_sn, p.v_sh, p.v_sb, box_tok, tok_first);
  }
  if (!ok) return TV_ERR_UNSUPPORTED;
  const bool two = p.R > HALF;
  const int tf = tok_first ? 1 : 0;
  if (dtype == TV_BF16) {
    if (paged) return two ? launch_t<__nv_bfloat16, 2, true>(p, mk, mv, box_tok, tf, st)
                          : launch_t<__nv_bfloat16, 1, true>(p, mk, mv, box_tok, tf, st);
    return two ? launch_t<__nv_bfloat16, 2, false>(p, mk, mv, box_tok, tf, st)
               : launch_t<__nv_bfloat16, 1, false>(p, mk, mv, box_tok, tf, st);
  }
  if (paged) return two ? launch_t<__half, 2, true>(p, mk, mv, box_tok, tf, st)
                        : launch_t<__half, 1, true>(p, mk, mv, box_tok, tf, st);
  return two ? launch_t<__half, 2, false>(p, mk, mv, box_tok, tf, st)
             : launch_t<__half, 1, false>(p, mk, mv, box_tok, tf, st);
}

}  // namespace tv
