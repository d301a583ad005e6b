// Verify attention, warp-MMA path (mma.sync m16n8k16, fp32 accumulate).
//
// One CTA = 4 warps = up to 64 query rows of one (batch, KV head) over one
// split of the keys.  Each warp computes 16 rows; with fewer than 64 rows per
// KV head (narrow trees) the warps split every key tile instead of computing
// padding rows: KS = 2 (up to 32 rows) or 4 (up to 16 rows) warps share a
// row group, each scoring its 1/KS of the tile's keys, and their (max, sum,
// O) are merged through shared memory at the end.  Query rows are (tree node, query head of the GQA group) pairs,
// r = node * G + g, so a KV tile staged in shared memory serves every head
// of the group: nothing is expanded per query head (the reference
// materialises repeat_kv copies, llama_target_model.py:795-796).
//
// Keys arrive in 64-key tiles by cp.async (16-byte chunks, zero-filled past
// the end or for missing pages), three tiles in flight.  For a paged cache every key
// looks up its physical page; the pool layout [page][kv_head][token][D] keeps
// a page's 16 tokens of one head contiguous, so one 64-key tile is four 4 KB
// runs.  Scores go through an online softmax in the exp2 domain; keys of the
// tree tail are gated by one bit per (node, key) instead of the reference's
// int8 [M, M] mask (tree_attention.py:449-460).
//
// This path serves narrow trees (fewer than 64 query rows per KV head) and
// every shape the tensor-memory path does not take.
#include "attn_epilogue.cuh"
#include "attn_kernels.cuh"

namespace tv {
namespace {

constexpr int BM = 64;      // query rows per CTA at KS = 1
constexpr int BN = 64;      // keys per tile
constexpr int NTHREADS = 128;
constexpr int STAGES = 3;

template <int D>
struct Geo {
  static constexpr int ROWB = D * 2;             // bytes per staged row
  static constexpr int CH = ROWB / 16;           // 16-byte chunks per row
  static constexpr int SW = CH < 8 ? CH : 8;     // swizzle period
  static __device__ __forceinline__ int swz(int row, int c) { return row * ROWB + ((c ^ (row & (SW - 1))) << 4); }
  static constexpr int Q_BYTES = BM * ROWB;
  static constexpr int T_BYTES = BN * ROWB;
  static constexpr int SMEM = Q_BYTES + 2 * STAGES * T_BYTES;
};

template <typename T, int D, bool PAGED>
__device__ __forceinline__ void load_kv_tile(const AttnParams& p, uint8_t* sK, uint8_t* sV, int b, int hk, int len,
                                             int tile, int tid) {
  using G = Geo<D>;
  const T* kb = static_cast<const T*>(p.k);
  const T* vb = static_cast<const T*>(p.v);
#pragma unroll
  for (int j = 0; j < (BN * G::CH) / NTHREADS; ++j) {
    const int idx = tid + j * NTHREADS;
    const int row = idx / G::CH;
    const int c = idx % G::CH;
    const int n = tile * BN + row;
    const T* ks = kb;
    const T* vs = vb;
    int bytes = 0;
    if (n < len) {
      if (PAGED) {
        const int page = p.pt[(int64_t)b * p.pt_sb + (n >> p.page_shift)];
        if (page >= 0 && page < p.num_pages) {
          const int off = n & ((1 << p.page_shift) - 1);
          ks = kb + (int64_t)page * p.k_sb + (int64_t)hk * p.k_sh + (int64_t)off * p.k_sn + c * 8;
          vs = vb + (int64_t)page * p.v_sb + (int64_t)hk * p.v_sh + (int64_t)off * p.v_sn + c * 8;
          bytes = 16;
        }
      } else {
        ks = kb + (int64_t)b * p.k_sb + (int64_t)n * p.k_sn + (int64_t)hk * p.k_sh + c * 8;
        vs = vb + (int64_t)b * p.v_sb + (int64_t)n * p.v_sn + (int64_t)hk * p.v_sh + c * 8;
        bytes = 16;
      }
    }
    cp_async16(smem_u32(sK + G::swz(row, c)), ks, bytes);
    cp_async16(smem_u32(sV + G::swz(row, c)), vs, bytes);
  }
}

// Split p into a pair of 16-bit values whose sum carries ~16 more mantissa bits.
template <typename T>
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  hi = Elem<T>::pack2(a, b);
  const T* h = reinterpret_cast<const T*>(&hi);
  lo = Elem<T>::pack2(a - Elem<T>::to_f(h[0]), b - Elem<T>::to_f(h[1]));
}

// PRECISE: the softmax weights enter the PV product as a hi + lo pair of
// 16-bit values (two MMAs) instead of one rounded value.  Rounding P to bf16
// alone costs up to 2^-9 * max|v| of absolute error per output, which matters
// when a row sees few keys; the pair brings it to ~2^-17.
template <typename T, int D, bool PAGED, bool PRECISE, int KS>
__global__ void __launch_bounds__(NTHREADS) attn_mma_kernel(const AttnParams p) {
  using G = Geo<D>;
  constexpr int RG = 4 / KS;          // row groups of 16 rows per CTA
  constexpr int BMK = 16 * RG;        // query rows per CTA
  constexpr int KW = BN / KS;         // keys of a tile scored by one warp
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + G::Q_BYTES;
  uint8_t* sV = sK + STAGES * G::T_BYTES;

  const int rb = blockIdx.x;
  const int bh = blockIdx.y;
  const int split = blockIdx.z;
  const int b = bh / p.Hkv;
  const int hk = bh - b * p.Hkv;
  int len = p.kv_lens ? p.kv_lens[b] : p.num_keys;
  len = len < 0 ? 0 : len;
  const int tail = len - p.mask_len;
  const int ntiles = (len + BN - 1) / BN;
  const int t0 = split * p.tiles_per_split;
  const int t1 = min(ntiles, t0 + p.tiles_per_split);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int gid = lane >> 2;
  const int tig = lane & 3;
  const int rg = warp % RG;           // this warp's row group
  const int kq = warp / RG;           // and its share of every key tile

  // ---- stage the 64 query rows of this CTA --------------------------------
  {
    const T* qb = static_cast<const T*>(p.q);
#pragma unroll
    for (int j = 0; j < (BMK * G::CH + NTHREADS - 1) / NTHREADS; ++j) {
      const int idx = tid + j * NTHREADS;
      if (idx >= BMK * G::CH) break;
      const int row = idx / G::CH;
      const int c = idx % G::CH;
      const int r = rb * BMK + row;
      const T* src = qb;
      int bytes = 0;
      if (r < p.R) {
        int m, h;
        row_coords(p, hk, r, m, h);
        src = qb + (int64_t)b * p.q_sb + (int64_t)m * p.q_sm + (int64_t)h * p.q_sh + c * 8;
        bytes = 16;
      }
      cp_async16(smem_u32(sQ + G::swz(row, c)), src, bytes);
    }
  }
  // tiles t0 and t0 + 1 in flight before the loop (one commit group each)
  if (t0 < t1) load_kv_tile<T, D, PAGED>(p, sK, sV, b, hk, len, t0, tid);
  cp_async_commit();
  if (t0 + 1 < t1) load_kv_tile<T, D, PAGED>(p, sK + G::T_BYTES, sV + G::T_BYTES, b, hk, len, t0 + 1, tid);
  cp_async_commit();

  // Rows held by this thread: its warp's row group's rows gid and gid + 8.
  const int r0 = rb * BMK + rg * 16 + gid;
  const int r1 = r0 + 8;
  const int m0 = min(r0, p.R - 1) / p.G;
  const int m1 = min(r1, p.R - 1) / p.G;
  const uint64_t* mrow0 = p.mask ? p.mask + (int64_t)b * p.mask_sb + (int64_t)m0 * p.mask_sm : nullptr;
  const uint64_t* mrow1 = p.mask ? p.mask + (int64_t)b * p.mask_sb + (int64_t)m1 * p.mask_sm : nullptr;

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float mx0 = -INFINITY, mx1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qf[D / 16][4];

  for (int t = t0; t < t1; ++t) {
    const int st = (t - t0) % STAGES;
    // Tile t + 2 into the stage tile t - 1 used (freed by the barrier that
    // ended the previous iteration); every iteration commits one group, so
    // waiting for all but the newest two leaves tile t landed.
    if (t + 2 < t1) {
      const int s2 = (t + 2 - t0) % STAGES;
      load_kv_tile<T, D, PAGED>(p, sK + s2 * G::T_BYTES, sV + s2 * G::T_BYTES, b, hk, len, t + 2, tid);
    }
    cp_async_commit();
    cp_async_wait<2>();
    __syncthreads();
    if (t == t0) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int row = rg * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = kk * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sQ + G::swz(row, c)), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    const uint8_t* tK = sK + st * G::T_BYTES;
    const uint8_t* tV = sV + st * G::T_BYTES;

    // ---- S = Q K^T (16 rows x KW keys per warp) ---------------------------
    float s[KW / 8][4];
#pragma unroll
    for (int i = 0; i < KW / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int nn = 0; nn < KW / 16; ++nn) {
        const int row = kq * KW + nn * 16 + (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(tK + G::swz(row, c)), b0, b1, b2, b3);
        Mma<T>::run(s[2 * nn], qf[kk], b0, b1);
        Mma<T>::run(s[2 * nn + 1], qf[kk], b2, b3);
      }
    }

    // ---- scale, bound and tree-mask the scores -----------------------------
    const int nbase = t * BN + kq * KW;
    const bool edge = (nbase + KW > len) || (nbase + KW > tail);
#pragma unroll
    for (int j = 0; j < KW / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * p.scale_log2;
        if (edge) {
          const int n = nbase + j * 8 + 2 * tig + (e & 1);
          if (n >= len) {
            x = -INFINITY;
          } else if (n >= tail) {
            const int rel = n - tail;
            const uint64_t* mr = (e < 2) ? mrow0 : mrow1;
            const uint64_t w = __ldg(mr + (rel >> 6));
            if (!((w >> (rel & 63)) & 1ull)) x = -INFINITY;
          }
        }
        s[j][e] = x;
      }
    }

    // ---- online softmax (exp2 domain) --------------------------------------
    float tmax0 = -INFINITY, tmax1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < KW / 8; ++j) {
      tmax0 = fmaxf(tmax0, fmaxf(s[j][0], s[j][1]));
      tmax1 = fmaxf(tmax1, fmaxf(s[j][2], s[j][3]));
    }
    tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, 1));
    tmax0 = fmaxf(tmax0, __shfl_xor_sync(0xffffffffu, tmax0, 2));
    tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, 1));
    tmax1 = fmaxf(tmax1, __shfl_xor_sync(0xffffffffu, tmax1, 2));
    const float nm0 = fmaxf(mx0, tmax0);
    const float nm1 = fmaxf(mx1, tmax1);
    const float use0 = nm0 == -INFINITY ? 0.f : nm0;
    const float use1 = nm1 == -INFINITY ? 0.f : nm1;
    const float a0 = fast_exp2(mx0 - use0);
    const float a1 = fast_exp2(mx1 - use1);
    mx0 = nm0;
    mx1 = nm1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < KW / 8; ++j) {
      s[j][0] = fast_exp2(s[j][0] - use0);
      s[j][1] = fast_exp2(s[j][1] - use0);
      s[j][2] = fast_exp2(s[j][2] - use1);
      s[j][3] = fast_exp2(s[j][3] - use1);
      ps0 += s[j][0] + s[j][1];
      ps1 += s[j][2] + s[j][3];
    }
    l0 = l0 * a0 + ps0;
    l1 = l1 * a1 + ps1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= a0;
      o[i][1] *= a0;
      o[i][2] *= a1;
      o[i][3] *= a1;
    }

    // ---- O += P V ------------------------------------------------------------
#pragma unroll
    for (int kk = 0; kk < KW / 16; ++kk) {
      uint32_t a[4], al[4];
      if (PRECISE) {
        split_pair<T>(s[2 * kk][0], s[2 * kk][1], a[0], al[0]);
        split_pair<T>(s[2 * kk][2], s[2 * kk][3], a[1], al[1]);
        split_pair<T>(s[2 * kk + 1][0], s[2 * kk + 1][1], a[2], al[2]);
        split_pair<T>(s[2 * kk + 1][2], s[2 * kk + 1][3], a[3], al[3]);
      } else {
        a[0] = Elem<T>::pack2(s[2 * kk][0], s[2 * kk][1]);
        a[1] = Elem<T>::pack2(s[2 * kk][2], s[2 * kk][3]);
        a[2] = Elem<T>::pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        a[3] = Elem<T>::pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
      }
#pragma unroll
      for (int dd = 0; dd < D / 16; ++dd) {
        const int row = kq * KW + kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = dd * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(tV + G::swz(row, c)), b0, b1, b2, b3);
        Mma<T>::run(o[2 * dd], a, b0, b1);
        Mma<T>::run(o[2 * dd + 1], a, b2, b3);
        if (PRECISE) {
          Mma<T>::run(o[2 * dd], al, b0, b1);
          Mma<T>::run(o[2 * dd + 1], al, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // ---- finish the rows -------------------------------------------------------
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  if (KS > 1) {
    // Merge the KS warps of each row group (same rows, disjoint keys): the
    // helpers leave (max, sum, O) in shared memory (the K/V stages are free
    // now), the first warp of the group folds them in.
    __syncthreads();
    float* xo = reinterpret_cast<float*>(sK);                       // [warp][lane][D / 2]
    float* xs = xo + NTHREADS * (D / 2);                            // [warp][lane][4]
    if (kq > 0) {
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<float4*>(xo + (warp * 32 + lane) * (D / 2) + 4 * i) =
            make_float4(o[i][0], o[i][1], o[i][2], o[i][3]);
      *reinterpret_cast<float4*>(xs + (warp * 32 + lane) * 4) = make_float4(mx0, mx1, l0, l1);
    }
    __syncthreads();
    if (kq == 0) {
#pragma unroll
      for (int q = 1; q < KS; ++q) {
        const int w2 = warp + q * RG;
        const float4 st2 = *reinterpret_cast<const float4*>(xs + (w2 * 32 + lane) * 4);
        const float n0 = fmaxf(mx0, st2.x), n1 = fmaxf(mx1, st2.y);
        const float u0 = n0 == -INFINITY ? 0.f : n0, u1 = n1 == -INFINITY ? 0.f : n1;
        const float a0 = fast_exp2(mx0 - u0), b0 = fast_exp2(st2.x - u0);
        const float a1 = fast_exp2(mx1 - u1), b1 = fast_exp2(st2.y - u1);
#pragma unroll
        for (int i = 0; i < D / 8; ++i) {
          const float4 v2 = *reinterpret_cast<const float4*>(xo + (w2 * 32 + lane) * (D / 2) + 4 * i);
          o[i][0] = o[i][0] * a0 + v2.x * b0;
          o[i][1] = o[i][1] * a0 + v2.y * b0;
          o[i][2] = o[i][2] * a1 + v2.z * b1;
          o[i][3] = o[i][3] * a1 + v2.w * b1;
        }
        l0 = l0 * a0 + st2.z * b0;
        l1 = l1 * a1 + st2.w * b1;
        mx0 = n0;
        mx1 = n1;
      }
    } else {
      return;                                                       // merged by the group's first warp
    }
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f;
  const float inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const float lse0 = l0 > 0.f ? (mx0 + __log2f(l0)) * kLn2 : -INFINITY;
  const float lse1 = l1 > 0.f ? (mx1 + __log2f(l1)) * kLn2 : -INFINITY;

  if (!p.part_o) {
    if (r0 < p.R) {
      int m, h;
      row_coords(p, hk, r0, m, h);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) store_out_pair<T>(p, b, m, h, i * 8 + 2 * tig, o[i][0] * inv0, o[i][1] * inv0);
      if (tig == 0) store_row_stats<T>(p, b, m, h, lse0);
    }
    if (r1 < p.R) {
      int m, h;
      row_coords(p, hk, r1, m, h);
#pragma unroll
      for (int i = 0; i < D / 8; ++i) store_out_pair<T>(p, b, m, h, i * 8 + 2 * tig, o[i][2] * inv1, o[i][3] * inv1);
      if (tig == 0) store_row_stats<T>(p, b, m, h, lse1);
    }
  } else {
    if (r0 < p.R) {
      float* dst = part_o_row(p, split, bh, r0, D);
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<float2*>(dst + i * 8 + 2 * tig) = make_float2(o[i][0] * inv0, o[i][1] * inv0);
      if (tig == 0) *part_lse_row(p, split, bh, r0) = lse0;
    }
    if (r1 < p.R) {
      float* dst = part_o_row(p, split, bh, r1, D);
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<float2*>(dst + i * 8 + 2 * tig) = make_float2(o[i][2] * inv1, o[i][3] * inv1);
      if (tig == 0) *part_lse_row(p, split, bh, r1) = lse1;
    }
  }
}

// Warps per row group: 4 for up to 16 rows per KV head, 2 for up to 32.
int key_split(int R) { return R <= 16 ? 4 : R <= 32 ? 2 : 1; }

template <typename T, int D, bool PAGED, bool PRECISE, int KS>
int launch_k(const AttnParams& p, cudaStream_t st) {
  constexpr int smem = Geo<D>::SMEM;
  static_assert(NTHREADS * (D / 2 + 4) * 4 <= 2 * STAGES * Geo<D>::T_BYTES, "merge scratch");
  auto kern = attn_mma_kernel<T, D, PAGED, PRECISE, KS>;
  const int rc_smem = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), smem);
  if (rc_smem != TV_OK) return rc_smem;
  constexpr int rows = 64 / KS;
  dim3 grid((p.R + rows - 1) / rows, p.B * p.Hkv, p.splits);
  kern<<<grid, NTHREADS, smem, st>>>(p);
  return check_launch();
}

template <typename T, int D, bool PAGED, bool PRECISE>
int launch_t(const AttnParams& p, cudaStream_t st) {
  switch (key_split(p.R)) {
    case 4: return launch_k<T, D, PAGED, PRECISE, 4>(p, st);
    case 2: return launch_k<T, D, PAGED, PRECISE, 2>(p, st);
    default: return launch_k<T, D, PAGED, PRECISE, 1>(p, st);
  }
}

template <typename T, int D>
int launch_d(const AttnParams& p, bool precise, cudaStream_t st) {
  const bool paged = p.pt != nullptr;
  if (precise) return paged ? launch_t<T, D, true, true>(p, st) : launch_t<T, D, false, true>(p, st);
  return paged ? launch_t<T, D, true, false>(p, st) : launch_t<T, D, false, false>(p, st);
}

template <typename T>
int launch_dtype(const AttnParams& p, int D, bool precise, cudaStream_t st) {
  switch (D) {
    case 32: return launch_d<T, 32>(p, precise, st);
    case 64: return launch_d<T, 64>(p, precise, st);
    case 128: return launch_d<T, 128>(p, precise, st);
    default: return TV_ERR_UNSUPPORTED;
  }
}

}  // namespace

int mma_tile_keys() { return BN; }
int mma_row_blocks(int R) {
  const int rows = 64 / key_split(R);
  return (R + rows - 1) / rows;
}

int launch_attn_mma(const AttnParams& p, int dtype, int D, bool precise, cudaStream_t st) {
  if (dtype == TV_BF16) return launch_dtype<__nv_bfloat16>(p, D, precise, st);
  if (dtype == TV_F16) return launch_dtype<__half>(p, D, precise, st);
  return TV_ERR_DTYPE;
}

}  // namespace tv
