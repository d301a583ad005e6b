// C ABI of verify attention: argument checks, split-KV planning, kernel
// selection, and the log-sum-exp merge kernels.
#include <string.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <queue>
#include <string>
#include <utility>
#include <vector>

#include "attn_epilogue.cuh"
#include "attn_kernels.cuh"

namespace tv {

static thread_local std::string g_last_cuda_error;

int record_cuda_error(cudaError_t e) {
  g_last_cuda_error = cudaGetErrorString(e);
  return TV_ERR_LAUNCH;
}

int ensure_dynamic_smem(const void* kernel, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;   // (kernel, device) -> limit set
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return record_cuda_error(e);
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = done.find({kernel, dev});
    if (it != done.end() && it->second >= bytes) return TV_OK;
  }
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return record_cuda_error(e);
  std::lock_guard<std::mutex> lock(mu);
  int& v = done[{kernel, dev}];
  if (bytes > v) v = bytes;
  return TV_OK;
}

namespace {

// ---- split combine: D/4 threads per query row, one float4 of O each --------
template <typename T, int D>
__global__ void __launch_bounds__(128) split_combine_kernel(const AttnParams p) {
  constexpr int TPR = D / 4;          // threads per row
  constexpr int RPB = 128 / TPR;      // rows per block
  const int q = threadIdx.x % TPR;
  const int64_t row = (int64_t)blockIdx.x * RPB + threadIdx.x / TPR;
  const int64_t total = (int64_t)p.B * p.Hkv * p.R;
  if (row >= total) return;
  const int bh = (int)(row / p.R);
  const int r = (int)(row - (int64_t)bh * p.R);
  const int b = bh / p.Hkv;
  const int hk = bh - b * p.Hkv;
  float4 o;
  float lse;
  combine_split_row<D>(p, bh, r, q, o, lse);
  int m, h;
  row_coords(p, hk, r, m, h);
  store_out_pair<T>(p, b, m, h, 4 * q, o.x, o.y);
  store_out_pair<T>(p, b, m, h, 4 * q + 2, o.z, o.w);
  if (q == 0) store_row_stats<T>(p, b, m, h, lse);
}

template <typename T>
__device__ __forceinline__ void store_plain(void* out, int64_t off, float v) {
  static_cast<T*>(out)[off] = Elem<T>::from_f(v);
}
template <>
__device__ __forceinline__ void store_plain<float>(void* out, int64_t off, float v) {
  static_cast<float*>(out)[off] = v;
}

// ---- generic merge of `parts` partials (split-KV or one per rank) -------------
template <typename OutT>
__global__ void __launch_bounds__(128) merge_parts_kernel(int parts, int64_t rows, int D, const float* po,
                                                          int64_t pso, const float* pl, int64_t psl, void* out,
                                                          float* out_lse) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 4 + warp;
  if (row >= rows) return;
  float mx = -INFINITY;
  for (int s = lane; s < parts; s += 32) mx = fmaxf(mx, pl[s * psl + row]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float wsum = 0.f;
  for (int s = 0; s < parts && mx != -INFINITY; ++s) {
    const float l = pl[s * psl + row];
    if (l != -INFINITY) wsum += expf(l - mx);
  }
  const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
  for (int d = lane; d < D; d += 32) {
    float acc = 0.f;
    for (int s = 0; s < parts && mx != -INFINITY; ++s) {
      const float l = pl[s * psl + row];
      if (l == -INFINITY) continue;
      acc += expf(l - mx) * po[s * pso + row * D + d];
    }
    store_plain<OutT>(out, row * D + d, acc * inv);
  }
  if (lane == 0 && out_lse) out_lse[row] = wsum > 0.f ? mx + logf(wsum) : -INFINITY;
}

bool stride_ok(int64_t s) { return (s % 8) == 0; }

constexpr int kPreciseMaxKeys = 4096;

int validate(const tv_attn_args* a) {
  if (!a) return TV_ERR_NULL;
  if (a->dtype != TV_BF16 && a->dtype != TV_F16) return TV_ERR_DTYPE;
  if (a->batch < 0 || a->rows < 0 || a->heads <= 0 || a->kv_heads <= 0) return TV_ERR_SHAPE;
  if (a->heads % a->kv_heads != 0) return TV_ERR_SHAPE;
  if (a->head_dim != 32 && a->head_dim != 64 && a->head_dim != 128) return TV_ERR_UNSUPPORTED;
  if (a->num_keys < 0 || a->mask_len < 0) return TV_ERR_SHAPE;
  if (a->batch == 0 || a->rows == 0) return TV_OK;
  if (!a->q || !a->out) return TV_ERR_NULL;
  if (a->num_keys > 0 && (!a->k || !a->v)) return TV_ERR_NULL;
  if (a->mask_len > 0 && !a->mask) return TV_ERR_NULL;
  if (!a->kv_lens && a->mask_len > a->num_keys) return TV_ERR_SHAPE;
  if (a->aux_lse && !a->weight) return TV_ERR_NULL;
  if (!aligned16(a->q) || !stride_ok(a->q_sb) || !stride_ok(a->q_sm) || !stride_ok(a->q_sh)) return TV_ERR_ALIGN;
  if (a->num_keys > 0) {
    if (!aligned16(a->k) || !aligned16(a->v)) return TV_ERR_ALIGN;
    if (!stride_ok(a->k_sb) || !stride_ok(a->k_sn) || !stride_ok(a->k_sh)) return TV_ERR_ALIGN;
    if (!stride_ok(a->v_sb) || !stride_ok(a->v_sn) || !stride_ok(a->v_sh)) return TV_ERR_ALIGN;
  }
  // Output rows are written two elements at a time.
  const size_t esz = a->out_f32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(a->out) % (2 * esz)) != 0) return TV_ERR_ALIGN;
  if ((a->o_sb | a->o_sm | a->o_sh) & 1) return TV_ERR_ALIGN;
  if (a->page_table) {
    if (a->page_size <= 0 || (a->page_size & (a->page_size - 1))) return TV_ERR_UNSUPPORTED;
    if (a->num_pages <= 0) return TV_ERR_SHAPE;
  }
  return TV_OK;
}

// Makespan, in tile-times, of base x splits tensor-memory CTAs (one per SM)
// dispatched split by split -- the split is the grid's slowest dimension, so
// every row-block CTA of split z starts before any of split z + 1 -- each
// taking its split's tiles plus a fixed cost: ~4 tiles for a CTA of the
// first wave (TMEM allocation, query staging, the first K/V tile from HBM)
// and ~12 for one that starts on an SM another CTA leaves (fitted to the
// measured multi-wave runs: 37 splits of config 2 in four waves, 171 of
// config 4).
double tc_makespan(int64_t base, int tiles, int tps) {
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < kNumSMs; ++i) free_at.push(0.0);
  double end = 0.0;
  const int splits = (tiles + tps - 1) / tps;
  for (int z = 0; z < splits; ++z) {
    const int t = tiles - z * tps < tps ? tiles - z * tps : tps;
    for (int64_t c = 0; c < base; ++c) {
      const double s = free_at.top();
      free_at.pop();
      const double e = s + t + (s == 0.0 ? 4.0 : 12.0);
      free_at.push(e);
      if (e > end) end = e;
    }
  }
  return end;
}

// Tiles per split for the tensor-memory kernel when `tps` (the plan below)
// leaves SMs idle: a last, shorter split whose CTAs fill the idle SMs and
// then the SMs its first CTAs leave can finish sooner (config 4, 128 nodes x
// GQA 4 = 32 row-block CTAs: 4 splits of 257 tiles use 128 of 148 SMs; 4 of
// 229 + one of 109 are predicted 10 % shorter).  Taken only for a predicted
// gain of 5 % or more; cached per (CTAs per split, tiles).
int tc_balance_tiles(int64_t base, int tiles, int tps) {
  static std::mutex mu;
  static std::map<std::pair<int64_t, int>, int> memo;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = memo.find({base, tiles});
    if (it != memo.end()) return it->second;
  }
  int best_tps = tps;
  const int64_t ctas = base * ((tiles + tps - 1) / tps);
  // Nothing to gain when the equal splits already fill 95 % of the SMs (a
  // 5 % gain is the bar below), or run in more than one wave.
  if (base > 0 && ctas <= kNumSMs && ctas * 20 < 19LL * kNumSMs) {
    const double cur = tc_makespan(base, tiles, tps);
    double best = cur;
    const int64_t max_splits = 2LL * kNumSMs / base;
    const int lo = max_splits > 0 ? (int)((tiles + max_splits - 1) / max_splits) : tps;
    for (int x = lo > 1 ? lo : 1; x < tps; ++x) {
      const int sx = (tiles + x - 1) / x;
      if (sx > 256 || base * sx > 2LL * kNumSMs) continue;
      const double m = tc_makespan(base, tiles, x);
      if (m < best) { best = m; best_tps = x; }
    }
    if (best > 0.95 * cur) best_tps = tps;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (memo.size() >= 4096) memo.clear();   // a long decode loop sees a new key count every 128 tokens
  memo[{base, tiles}] = best_tps;
  return best_tps;
}

struct Plan {
  bool tc;
  int tile;
  int splits;
  int tiles_per_split;
};

Plan plan(const tv_attn_args* a) {
  const int D = a->head_dim;
  const int G = a->heads / a->kv_heads;
  const int R = a->rows * G;
  const bool paged = a->page_table != nullptr;
  int shift = 0;
  if (paged) while ((1 << shift) < a->page_size) ++shift;
  Plan pl;
  const int sel = a->kernel & 15;
  // The tensor-memory kernel takes long, uniform-length key ranges (any
  // length: it zeroes the unused rows of a last page that ends mid-tile).
  pl.tc = (sel != 1) && !(a->kernel & 16) && !a->kv_lens && a->num_keys > kPreciseMaxKeys &&
          tc_supported(a->dtype, D, R, paged, shift);
  pl.tile = pl.tc ? tc_tile_keys() : mma_tile_keys();
  const int row_blocks = pl.tc ? tc_row_blocks(R) : mma_row_blocks(R);
  const int64_t base = (int64_t)row_blocks * a->batch * a->kv_heads;
  const int tiles = (a->num_keys + pl.tile - 1) / pl.tile;
  int splits = a->num_splits;
  if (splits <= 0) {
    if (pl.tc) {
      // Tensor-memory CTAs fill an SM each (one per SM): one wave of at most
      // 148 (config 2: 16 row-block CTAs x 9 splits = 144).  Only when that
      // wave would leave more than a quarter of the SMs idle (few splits of
      // many row blocks, e.g. batch 4 x 3 row blocks x 8 KV heads = 96) may
      // the CTAs run in more waves: waves x (tiles per CTA + a fixed cost of
      // about 16 tiles for the pipeline fill, drain and epilogue) decides.
      // Measured: many short CTAs in several waves lose to one full wave.
      splits = (int)(kNumSMs / base);
      if (splits < 1) splits = 1;
      if (base * splits * 4 < 3LL * kNumSMs) {
        int64_t best = INT64_MAX;
        for (int s = 1; s <= 256 && s <= tiles && base * s <= 4LL * kNumSMs; ++s) {
          const int64_t waves = (base * s + kNumSMs - 1) / kNumSMs;
          const int64_t cost = waves * ((tiles + s - 1) / s + 16);
          if (cost < best) { best = cost; splits = s; }
        }
      }
    } else {
      // The warp-MMA CTAs (112 KB of shared memory) run two per SM: one wave
      // of 2 x 148 (measured: 37 splits of 8 row-block CTAs beat 74 by 10 %).
      splits = (int)(2LL * kNumSMs / base);
      if (splits < 1) splits = 1;
    }
  }
  if (splits > tiles) splits = tiles;
  if (splits > 256) splits = 256;
  if (splits < 1) splits = 1;
  pl.tiles_per_split = tiles > 0 ? (tiles + splits - 1) / splits : 1;
  if (pl.tc && a->num_splits <= 0 && tiles > 0)
    pl.tiles_per_split = tc_balance_tiles(base, tiles, pl.tiles_per_split);
  pl.splits = tiles > 0 ? (tiles + pl.tiles_per_split - 1) / pl.tiles_per_split : 1;
  return pl;
}

// kernel selector 2 asks for the tensor-memory kernel and nothing else.
bool plan_allowed(const tv_attn_args* a, const Plan& pl) { return (a->kernel & 15) != 2 || pl.tc; }

// Bytes of `splits` partials: O [splits][rows][D] fp32 (256-byte aligned end),
// then LSE [splits][rows] fp32.
size_t partial_bytes(const tv_attn_args* a, int splits) {
  const int G = a->heads / a->kv_heads;
  const int64_t rows = (int64_t)a->batch * a->kv_heads * a->rows * G;
  const size_t o = (size_t)splits * rows * a->head_dim * sizeof(float);
  const size_t l = (size_t)splits * rows * sizeof(float);
  return ((o + 255) & ~size_t(255)) + l;
}

size_t workspace_for(const tv_attn_args* a, const Plan& pl) {
  return pl.splits <= 1 ? 0 : partial_bytes(a, pl.splits);
}

// Kernel parameters of a validated request; partials (when `partials`) in
// a->workspace.
void fill_params(const tv_attn_args* a, const Plan& pl, bool partials, AttnParams& p) {
  memset(&p, 0, sizeof(p));
  p.q = a->q;
  p.q_sb = a->q_sb; p.q_sm = a->q_sm; p.q_sh = a->q_sh;
  p.k = a->k ? a->k : a->q;
  p.v = a->v ? a->v : a->q;
  p.k_sb = a->k_sb; p.k_sn = a->k_sn; p.k_sh = a->k_sh;
  p.v_sb = a->v_sb; p.v_sn = a->v_sn; p.v_sh = a->v_sh;
  p.pt = a->page_table;
  p.pt_sb = a->pt_sb;
  p.page_shift = 0;
  if (a->page_table) while ((1 << p.page_shift) < a->page_size) ++p.page_shift;
  p.num_pages = a->num_pages;
  p.kv_lens = a->kv_lens;
  p.num_keys = a->num_keys;
  p.mask_len = a->mask_len;
  p.mask = a->mask;
  p.mask_sb = a->mask_sb; p.mask_sm = a->mask_sm;
  p.mfull = a->mask ? a->mask_words_full : nullptr;
  p.mfull_sb = a->mask_words_full_sb;
  p.B = a->batch; p.M = a->rows; p.H = a->heads; p.Hkv = a->kv_heads;
  p.G = a->heads / a->kv_heads;
  p.R = a->rows * p.G;
  p.scale_log2 = a->scale * kLog2e;
  p.splits = pl.splits;
  p.tiles_per_split = pl.tiles_per_split;
  p.out = a->out;
  p.o_sb = a->o_sb; p.o_sm = a->o_sm; p.o_sh = a->o_sh;
  p.out_f32 = a->out_f32;
  p.lse = a->lse;
  p.lse_sb = a->lse_sb; p.lse_sm = a->lse_sm; p.lse_sh = a->lse_sh;
  p.aux = a->aux_lse;
  p.aux_sb = a->aux_sb; p.aux_sm = a->aux_sm; p.aux_sh = a->aux_sh;
  p.weight = a->weight;
  p.w_sb = a->w_sb; p.w_sm = a->w_sm; p.w_sh = a->w_sh;
  p.err = a->status;
  if (partials) {
    const int64_t rows = (int64_t)p.B * p.Hkv * p.R;
    const size_t o = (size_t)pl.splits * rows * a->head_dim * sizeof(float);
    p.part_o = static_cast<float*>(a->workspace);
    p.part_lse = reinterpret_cast<float*>(static_cast<char*>(a->workspace) + ((o + 255) & ~size_t(255)));
  }
}

// Short key ranges take the split-P PV product (see attn_mma.cu); long ones
// average the bf16 rounding of P away.  Bit 4 of `kernel` forces it.
int launch_attention(const tv_attn_args* a, const Plan& pl, const AttnParams& p, cudaStream_t st) {
  const bool precise = (a->kernel & 16) || a->num_keys <= kPreciseMaxKeys;
  return pl.tc ? launch_attn_tc(p, a->dtype, a->head_dim, a->kernel, st)
               : launch_attn_mma(p, a->dtype, a->head_dim, precise, st);
}

}  // namespace

int launch_split_combine(const AttnParams& p, int dtype, int D, cudaStream_t st) {
  const int64_t rows = (int64_t)p.B * p.Hkv * p.R;
  const int64_t rows_per_block = 128 / (D / 4);
  dim3 grid((unsigned)((rows + rows_per_block - 1) / rows_per_block));
  if (dtype == TV_BF16) {
    if (D == 128) split_combine_kernel<__nv_bfloat16, 128><<<grid, 128, 0, st>>>(p);
    else if (D == 64) split_combine_kernel<__nv_bfloat16, 64><<<grid, 128, 0, st>>>(p);
    else split_combine_kernel<__nv_bfloat16, 32><<<grid, 128, 0, st>>>(p);
  } else {
    if (D == 128) split_combine_kernel<__half, 128><<<grid, 128, 0, st>>>(p);
    else if (D == 64) split_combine_kernel<__half, 64><<<grid, 128, 0, st>>>(p);
    else split_combine_kernel<__half, 32><<<grid, 128, 0, st>>>(p);
  }
  return check_launch();
}

}  // namespace tv

using namespace tv;

extern "C" {

const char* tv_status_string(int s) {
  switch (s) {
    case TV_OK: return "ok";
    case TV_ERR_SHAPE: return "inconsistent or unsupported sizes";
    case TV_ERR_DTYPE: return "unsupported element type";
    case TV_ERR_ALIGN: return "pointer or stride not 16-byte aligned";
    case TV_ERR_LAUNCH: return "CUDA launch or runtime error";
    case TV_ERR_WORKSPACE: return "workspace missing or too small";
    case TV_ERR_INPUT: return "invalid input values";
    case TV_ERR_UNSUPPORTED: return "request not supported by this build";
    case TV_ERR_NULL: return "required pointer is NULL";
    default: return "unknown status";
  }
}

const char* tv_version(void) { return "specverify 0.1 sm_100a"; }

const char* tv_last_cuda_error(void) { return g_last_cuda_error.c_str(); }

int tv_attn_workspace_size(const tv_attn_args* a, size_t* bytes) {
  if (!bytes) return TV_ERR_NULL;
  *bytes = 0;
  const int v = validate(a);
  if (v != TV_OK) return v;
  if (a->batch == 0 || a->rows == 0) return TV_OK;
  const Plan pl = plan(a);
  if (!plan_allowed(a, pl)) return TV_ERR_UNSUPPORTED;
  *bytes = workspace_for(a, pl);
  return TV_OK;
}

int tv_verify_attn(const tv_attn_args* a, void* stream) {
  const int v = validate(a);
  if (v != TV_OK) return v;
  if (a->batch == 0 || a->rows == 0) return TV_OK;
  const Plan pl = plan(a);
  if (!plan_allowed(a, pl)) return TV_ERR_UNSUPPORTED;
  const size_t need = workspace_for(a, pl);
  if (need > 0 && (!a->workspace || a->workspace_bytes < need)) return TV_ERR_WORKSPACE;
  if (need > 0 && !aligned16(a->workspace)) return TV_ERR_ALIGN;
  AttnParams p;
  fill_params(a, pl, pl.splits > 1, p);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int rc = launch_attention(a, pl, p, st);
  if (rc != TV_OK) return rc;
  if (pl.splits > 1) rc = launch_split_combine(p, a->dtype, a->head_dim, st);
  return rc;
}

int tv_attn_describe(const tv_attn_args* a, int32_t* info) {
  if (!info) return TV_ERR_NULL;
  info[0] = info[1] = info[2] = info[3] = 0;
  const int v = validate(a);
  if (v != TV_OK) return v;
  if (a->batch == 0 || a->rows == 0) return TV_OK;
  const Plan pl = plan(a);
  if (!plan_allowed(a, pl)) return TV_ERR_UNSUPPORTED;
  AttnParams p;
  fill_params(a, pl, pl.splits > 1, p);
  info[0] = pl.tc ? 2 : 1;
  info[1] = pl.splits;
  info[2] = pl.tc && a->page_table ? attn_tc_wide(p, a->dtype, a->kernel) : 0;
  info[3] = pl.tc ? 0 : ((a->kernel & 16) || a->num_keys <= kPreciseMaxKeys ? 1 : 0);
  return TV_OK;
}

int tv_verify_attn_sharded_workspace_size(const tv_attn_args* a, size_t* bytes) {
  if (!bytes) return TV_ERR_NULL;
  *bytes = 0;
  const int v = validate(a);
  if (v != TV_OK) return v;
  if (a->batch == 0 || a->rows == 0) return TV_OK;
  const Plan pl = plan(a);
  if (!plan_allowed(a, pl)) return TV_ERR_UNSUPPORTED;
  *bytes = partial_bytes(a, pl.splits);
  return TV_OK;
}

int tv_verify_attn_sharded(const tv_attn_args* a, int32_t world, int32_t rank, const void* const* bases,
                           int64_t exchange_bytes, void* stream) {
  const int v = validate(a);
  if (v != TV_OK) return v;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) return TV_ERR_SHAPE;
  if (!bases) return TV_ERR_NULL;
  for (int r = 0; r < world; ++r) {
    if (!bases[r]) return TV_ERR_NULL;
    if (!aligned16(bases[r])) return TV_ERR_ALIGN;
  }
  if (a->batch == 0 || a->rows == 0) return TV_OK;
  // The buffers' layout (slots, step counts per block of the exchange grid)
  // follows from (world, rows, head_dim): a buffer made for another shape
  // would take stores past its end or desynchronise the step counts.
  if (exchange_bytes != sharded_exchange_bytes(world, (int64_t)a->batch * a->rows * a->heads, a->head_dim))
    return TV_ERR_WORKSPACE;
  const Plan pl = plan(a);
  if (!plan_allowed(a, pl)) return TV_ERR_UNSUPPORTED;
  const size_t need = partial_bytes(a, pl.splits);
  if (!a->workspace || a->workspace_bytes < need) return TV_ERR_WORKSPACE;
  if (!aligned16(a->workspace)) return TV_ERR_ALIGN;
  AttnParams p;
  fill_params(a, pl, true, p);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int rc = launch_attention(a, pl, p, st);
  if (rc != TV_OK) return rc;
  // Exchange mode: bit 5 owner, bit 6 push to all; by default push below four
  // ranks, owner from four on (push sends 2 (W-1) partials per rank).
  const bool owned = (a->kernel & 32) ? true : (a->kernel & 64) ? false : world >= 4;
  return launch_sharded_combine(p, a->dtype, a->head_dim, world, rank, bases, owned, st);
}

int tv_merge_partials(int32_t parts, int64_t rows, int32_t head_dim, const float* parts_o, int64_t part_stride_o,
                      const float* parts_lse, int64_t part_stride_lse, int32_t out_dtype, void* out, float* out_lse,
                      void* stream) {
  if (parts <= 0 || rows < 0 || head_dim <= 0) return TV_ERR_SHAPE;
  if (rows == 0) return TV_OK;
  if (!parts_o || !parts_lse || !out) return TV_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  dim3 grid((unsigned)((rows + 3) / 4));
  switch (out_dtype) {
    case TV_BF16:
      merge_parts_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(parts, rows, head_dim, parts_o, part_stride_o,
                                                              parts_lse, part_stride_lse, out, out_lse);
      break;
    case TV_F16:
      merge_parts_kernel<__half><<<grid, 128, 0, st>>>(parts, rows, head_dim, parts_o, part_stride_o, parts_lse,
                                                       part_stride_lse, out, out_lse);
      break;
    case TV_F32:
      merge_parts_kernel<float><<<grid, 128, 0, st>>>(parts, rows, head_dim, parts_o, part_stride_o, parts_lse,
                                                      part_stride_lse, out, out_lse);
      break;
    default: return TV_ERR_DTYPE;
  }
  return check_launch();
}

}  // extern "C"
