// lm_head GEMM with the acceptance scan in its epilogue (sm_100a): the step
// after the verify attention, logits = lm_head(hidden) (diffspec_model.py:
// 229-231) and the per-node argmax / sample of verify_new
// (tree_verification.py:100-162), without ever writing the [rows, vocab]
// logits.
//
// A persistent CTA per SM walks 224-token vocabulary tiles.  For each tile
// the weight rows stream through a 5-stage shared-memory ring in 64-wide K
// chunks (TMA, 128-byte swizzle) together with the matching chunk of the
// hidden rows (at most 128, zero-padded by TMA), and one thread issues
// tcgen05.mma (M = 128, N = 224, K = 16) into one of two tensor-memory
// accumulators.  Four epilogue warps read the other accumulator (one row per
// thread), round each logit to the element type as the reference's logits
// are, add Gumbel noise when sampling, and keep each row's best (score,
// index) over all of the CTA's tiles -- one partial per (row, CTA) for the
// acceptance stage to reduce.
//
//   warp 0   TMA producer (the stage's two boxes from lane it mod 32)
//   warp 1   MMA issuer (one thread)
//   warps 2-5  epilogue (TMEM lane quarter w mod 4)
//
// The weight is read once from HBM: the kernel is bound by HBM bandwidth.
// Every mbarrier wait is bounded (2 s) and raises an abort flag on expiry.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "accept_common.cuh"
#include "sm100.cuh"

namespace tv {
namespace {

using namespace sm100;

constexpr int MR = 128;                  // hidden rows per MMA (zero-padded)
constexpr int NT = 224;                  // vocabulary rows per tile (MMA N)
constexpr int BK = 64;                   // K per stage (128 bytes of 16-bit values)
constexpr int A_BYTES = MR * 128;        // 16 KB
constexpr int B_BYTES = NT * 128;        // 28 KB
constexpr int STAGE = A_BYTES + B_BYTES; // 44 KB
constexpr int NSTAGE = 5;
constexpr int ACC_COLS = 256;            // accumulator stride in TMEM columns
constexpr int THREADS = 192;
constexpr int SMEM_BYTES = NSTAGE * STAGE + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct Bars {
  uint64_t full[NSTAGE];
  uint64_t empty[NSTAGE];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem;
  int abort;
};

template <typename T>
__device__ __forceinline__ float round_to(float x);
template <>
__device__ __forceinline__ float round_to<__nv_bfloat16>(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
template <>
__device__ __forceinline__ float round_to<__half>(float x) { return __half2float(__float2half_rn(x)); }

__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) { return smem_desc_sw128(saddr, 16, 1024); }

template <typename T, bool SAMPLE>
__global__ void __launch_bounds__(THREADS, 1)
    lmhead_scan_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, int rows,
                       int hidden, int vocab, int tiles, float inv_t, uint64_t seed, uint64_t offset, float* part_v,
                       int* part_i, int* err) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  if ((smem_u32(smem_raw) & 1023u) != 0) {
    if (threadIdx.x == 0 && err) atomicExch(err, 7);
    return;
  }
  Bars* bars = reinterpret_cast<Bars*>(smem_raw + NSTAGE * STAGE);
  volatile int* abort = &bars->abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = hidden / BK;
  // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars->acc_full[b], 1);
      mbar_init(&bars->acc_empty[b], 4);
    }
    bars->abort = 0;
    mbar_fence_init();
  }
  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmx);
      prefetch_tmap(&tmw);
    }
    __syncwarp();
    tmem_alloc(&bars->tmem, 2 * ACC_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem;

  if (warp == 0) {
    // ---------------------------------------------------------------- producer
    const int total = my_tiles * nk;
    bool failed = false;
    int it = 0;
    for (; it < total; ++it) {
      const int s = it % NSTAGE;
      int go = 1;
      if (it >= NSTAGE && lane == 0 && !mbar_wait(&bars->empty[s], ((it / NSTAGE) & 1) ^ 1, abort)) go = *abort ? 0 : -1;
      go = __shfl_sync(0xffffffffu, go, 0);
      if (go <= 0) {
        failed = go < 0;
        break;
      }
      const int tile = blockIdx.x + (it / nk) * gridDim.x;
      const int kc = it % nk;
      if (lane == (it & 31)) {       // a lane keeps about one box in flight: rotate
        uint8_t* st = smem_raw + s * STAGE;
        mbar_arrive_expect_tx(&bars->full[s], STAGE);
        tma_load_2d(st, &tmx, &bars->full[s], kc * BK, 0);
        tma_load_2d(st + A_BYTES, &tmw, &bars->full[s], kc * BK, tile * NT);
      }
      __syncwarp();
    }
    if (lane == 0) {
      if (failed) {
        bars->abort = 1;
        if (err) atomicExch(err, 1);
      }
      if (*abort) {
        // loads in flight land before shared memory is released
        volatile int keep_waiting = 0;
        for (int j = it > NSTAGE ? it - NSTAGE : 0; j < it; ++j)
          mbar_wait(&bars->full[j % NSTAGE], (j / NSTAGE) & 1, &keep_waiting, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      constexpr uint32_t idesc = idesc_f16(fmt, MR, NT, 0);
      bool ok = true;
      int it = 0;
      for (int ti = 0; ok && ti < my_tiles; ++ti) {
        const int ab = ti & 1;
        // the epilogue has read this accumulator's previous tile (ti - 2)
        if (ti >= 2 && !mbar_wait(&bars->acc_empty[ab], ((ti >> 1) & 1) ^ 1, abort)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(ab * ACC_COLS);
        for (int kc = 0; kc < nk; ++kc, ++it) {
          const int s = it % NSTAGE;
          if (!mbar_wait(&bars->full[s], (it / NSTAGE) & 1, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_u32(smem_raw + s * STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            mma_ss(d, desc_kmajor(a0 + kk * 32), desc_kmajor(a0 + A_BYTES + kk * 32), idesc, (kc | kk) ? 1u : 0u);
          tc_commit(&bars->empty[s]);
        }
        if (ok) tc_commit(&bars->acc_full[ab]);
      }
      if (!ok) {
        bars->abort = 1;
        if (err) atomicExch(err, 2);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q4 = warp & 3;
    const int r = q4 * 32 + lane;               // hidden row = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(q4 * 32) << 16);
    bool ok = true;
    // one running best per row over all of this CTA's tiles: one partial per
    // (row, CTA) for the acceptance stage
    acc::Best best{-INFINITY, 0x7fffffff};
    for (int ti = 0; ti < my_tiles; ++ti) {
      const int ab = ti & 1;
      const int tile = blockIdx.x + ti * gridDim.x;
      if (!__all_sync(0xffffffffu, mbar_wait(&bars->acc_full[ab], (ti >> 1) & 1, abort))) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < NT / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_base + (uint32_t)(ab * ACC_COLS + c * 32), v);
        tmem_wait_ld();
        const int j0 = tile * NT + c * 32;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          const int j = j0 + k;
          float x = round_to<T>(__uint_as_float(v[k]));
          if (SAMPLE) x = x * inv_t + acc::gumbel(seed, offset, r, j);
          if (j < vocab) acc::take(best, x, j);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[ab]);
    }
    if (r < rows) {
      part_v[(int64_t)r * gridDim.x + blockIdx.x] = best.v;
      part_i[(int64_t)r * gridDim.x + blockIdx.x] = best.i;
    }
    if (!ok) {
      bars->abort = 1;
      if (err) atomicExch(err, 3);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * ACC_COLS);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// [rows_total, K] row-major 16-bit matrix, box = 64 x box_rows, 128-byte swizzle.
bool make_map_2d(CUtensorMap* map, int dtype, const void* base, uint64_t k, uint64_t rows_total, int64_t row_stride,
                 uint32_t box_rows) {
  auto enc = encoder();
  if (!enc) return false;
  const CUtensorMapDataType dt = dtype == TV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {k, rows_total};
  cuuint64_t strides[1] = {(cuuint64_t)row_stride * 2};
  cuuint32_t box[2] = {BK, box_rows}, estr[2] = {1, 1};
  return enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int tiles_for(int vocab) { return (vocab + NT - 1) / NT; }
// persistent CTAs: one per SM, at most one per tile; one partial per (row, CTA)
int grid_for(int vocab) {
  const int t = tiles_for(vocab);
  return t < kNumSMs ? t : kNumSMs;
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" {

int tv_lmhead_accept_workspace_size(const tv_lmhead_args* a, size_t* bytes) {
  if (!a || !bytes) return TV_ERR_NULL;
  const int rows = a->rows > 0 ? a->rows : 0;
  const int parts = a->vocab > 0 ? grid_for(a->vocab) : 0;
  // partial scores, partial indices, then a 16-byte-aligned status word
  *bytes = (((size_t)rows * parts * (sizeof(float) + sizeof(int)) + 15) & ~size_t(15)) + 64;
  return TV_OK;
}

int tv_lmhead_accept(const tv_lmhead_args* a, void* stream) {
  if (!a) return TV_ERR_NULL;
  if (a->mode != 0 && a->mode != 1) return TV_ERR_INPUT;
  if (a->mode == 1 && !(a->temperature > 0.f)) return TV_ERR_INPUT;
  if (a->rows < 1 || a->rows > MR || a->vocab < 1 || a->hidden < BK || (a->hidden % BK) != 0) return TV_ERR_SHAPE;
  if (a->dtype != TV_BF16 && a->dtype != TV_F16) return TV_ERR_DTYPE;
  if (!a->x || !a->weight || !a->next_tokens) return TV_ERR_NULL;
  if (a->draft && (!a->pos || !a->result || (a->rows > 1 && !a->parent))) return TV_ERR_NULL;
  if (a->max_depth < 0) return TV_ERR_SHAPE;
  if (a->x_sm < a->hidden || a->w_sv < a->hidden) return TV_ERR_SHAPE;
  if (!aligned16(a->x) || !aligned16(a->weight) || (a->x_sm % 8) != 0 || (a->w_sv % 8) != 0) return TV_ERR_ALIGN;
  const int tiles = tiles_for(a->vocab);
  size_t need = 0;
  tv_lmhead_accept_workspace_size(a, &need);
  if (!a->workspace || a->workspace_bytes < need) return TV_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(a->workspace) & 15) != 0) return TV_ERR_ALIGN;
  const int grid = grid_for(a->vocab);
  float* pv = static_cast<float*>(a->workspace);
  int* pi = reinterpret_cast<int*>(pv + (size_t)a->rows * grid);
  int* err = reinterpret_cast<int*>(static_cast<uint8_t*>(a->workspace) +
                                    (((size_t)a->rows * grid * (sizeof(float) + sizeof(int)) + 15) & ~size_t(15)));
  CUtensorMap mx, mw;
  if (!make_map_2d(&mx, a->dtype, a->x, (uint64_t)a->hidden, (uint64_t)a->rows, a->x_sm, MR) ||
      !make_map_2d(&mw, a->dtype, a->weight, (uint64_t)a->hidden, (uint64_t)a->vocab, a->w_sv, NT))
    return TV_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const cudaError_t me = cudaMemsetAsync(err, 0, sizeof(int), st);
  if (me != cudaSuccess) return record_cuda_error(me);
  const float inv_t = a->mode == 1 ? 1.0f / a->temperature : 1.0f;
#define TV_LMHEAD(TT, SS)                                                                                     \
  do {                                                                                                        \
    auto kern = lmhead_scan_kernel<TT, SS>;                                                                   \
    const int rc_smem = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), SMEM_BYTES);                 \
    if (rc_smem != TV_OK) return rc_smem;                                                                     \
    kern<<<grid, THREADS, SMEM_BYTES, st>>>(mx, mw, a->rows, a->hidden, a->vocab, tiles, inv_t, a->seed,      \
                                            a->offset, pv, pi, err);                                          \
  } while (0)
  if (a->dtype == TV_BF16) {
    if (a->mode == 1) TV_LMHEAD(__nv_bfloat16, true);
    else TV_LMHEAD(__nv_bfloat16, false);
  } else {
    if (a->mode == 1) TV_LMHEAD(__half, true);
    else TV_LMHEAD(__half, false);
  }
#undef TV_LMHEAD
  const int rc = check_launch();
  if (rc != TV_OK) return rc;
  return launch_accept_decide(a->rows, grid, pv, pi, nullptr, a->draft, a->parent, a->pos, a->max_depth,
                              a->next_tokens, a->result, err, st);
}

}  // extern "C"
