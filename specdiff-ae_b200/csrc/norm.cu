// Row-wise elementwise work of the target's decoder layers around the verify
// path, one launch each: LlamaRMSNorm (runtime/llama_target_model.py:124-138)
// and the SwiGLU gate act_fn(gate) * up of LlamaMLP (:506-538), with the
// reference's roundings (fp32 statistics, the normalised row rounded to the
// element type before the weight multiply; silu rounded before the product).
//
// One CTA per row for the norm (the row's sum of squares is a block
// reduction); the gate is a flat grid over 8-element chunks.  Rows are read
// as 16-byte vectors: columns a multiple of 8, rows 16-byte aligned.
#include "common.cuh"
#include "specverify.h"

namespace tv {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
  for (int k = 0; k < 8; ++k) f[k] = Elem<T>::to_f(e[k]);
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* f) {
  uint4 u;
  uint32_t* w = reinterpret_cast<uint32_t*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) w[k] = Elem<T>::pack2(f[2 * k], f[2 * k + 1]);
  return u;
}

template <typename T>
__device__ __forceinline__ float round_to(float x) {
  return Elem<T>::to_f(Elem<T>::from_f(x));
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const T* __restrict__ x, int64_t xs,
                                                                const T* __restrict__ w, T* __restrict__ y,
                                                                int64_t ys, int cols, float eps) {
  const T* xr = x + (int64_t)blockIdx.x * xs;
  T* yr = y + (int64_t)blockIdx.x * ys;
  float ss = 0.f;
  for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
    float f[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(xr + c), f);
#pragma unroll
    for (int k = 0; k < 8; ++k) ss = fmaf(f[k], f[k], ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  __shared__ float part[kNormThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kNormThreads / 32; ++i) tot += part[i];
  const float inv = rsqrtf(tot / (float)cols + eps);
  for (int c = threadIdx.x * 8; c < cols; c += kNormThreads * 8) {
    float f[8], g[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(xr + c), f);
    unpack8<T>(*reinterpret_cast<const uint4*>(w + c), g);
#pragma unroll
    for (int k = 0; k < 8; ++k) f[k] = round_to<T>(f[k] * inv) * g[k];
    *reinterpret_cast<uint4*>(yr + c) = pack8<T>(f);
  }
}

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, int64_t in_s, T* __restrict__ y,
                                int64_t out_s, int rows, int cols) {
  const int chunks = cols / 8;
  const int64_t n = (int64_t)rows * chunks;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e / chunks;
    const int c = (int)(e - r * chunks) * 8;
    float a[8], b[8];
    unpack8<T>(*reinterpret_cast<const uint4*>(g + r * in_s + c), a);
    unpack8<T>(*reinterpret_cast<const uint4*>(u + r * in_s + c), b);
#pragma unroll
    for (int k = 0; k < 8; ++k) a[k] = round_to<T>(a[k] / (1.0f + expf(-a[k]))) * b[k];
    *reinterpret_cast<uint4*>(y + r * out_s + c) = pack8<T>(a);
  }
}

bool vec_ok(const void* p, int64_t stride) {
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (stride % 8) == 0;
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" {

int tv_rms_norm(const void* x, int64_t x_row_stride, const void* weight, void* y, int64_t y_row_stride,
                int32_t rows, int32_t cols, float eps, int32_t dtype, void* stream) {
  if (rows < 0 || cols <= 0 || (cols % 8) != 0) return TV_ERR_SHAPE;
  if (dtype != TV_BF16 && dtype != TV_F16) return TV_ERR_DTYPE;
  if (rows == 0) return TV_OK;
  if (!x || !weight || !y) return TV_ERR_NULL;
  if (!vec_ok(x, x_row_stride) || !vec_ok(y, y_row_stride) || !vec_ok(weight, 0)) return TV_ERR_ALIGN;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TV_BF16)
    rms_norm_kernel<__nv_bfloat16><<<rows, kNormThreads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(x), x_row_stride, static_cast<const __nv_bfloat16*>(weight),
        static_cast<__nv_bfloat16*>(y), y_row_stride, cols, eps);
  else
    rms_norm_kernel<__half><<<rows, kNormThreads, 0, st>>>(static_cast<const __half*>(x), x_row_stride,
                                                           static_cast<const __half*>(weight),
                                                           static_cast<__half*>(y), y_row_stride, cols, eps);
  return check_launch();
}

int tv_silu_mul(const void* gate, const void* up, int64_t in_row_stride, void* out, int64_t out_row_stride,
                int32_t rows, int32_t cols, int32_t dtype, void* stream) {
  if (rows < 0 || cols <= 0 || (cols % 8) != 0) return TV_ERR_SHAPE;
  if (dtype != TV_BF16 && dtype != TV_F16) return TV_ERR_DTYPE;
  if (rows == 0) return TV_OK;
  if (!gate || !up || !out) return TV_ERR_NULL;
  if (!vec_ok(gate, in_row_stride) || !vec_ok(up, in_row_stride) || !vec_ok(out, out_row_stride))
    return TV_ERR_ALIGN;
  const int64_t n = (int64_t)rows * (cols / 8);
  const int threads = 256;
  const int64_t want = (n + threads - 1) / threads;
  const int blocks = (int)(want < 4 * kNumSMs ? want : 4 * kNumSMs);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TV_BF16)
    silu_mul_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
        static_cast<const __nv_bfloat16*>(gate), static_cast<const __nv_bfloat16*>(up), in_row_stride,
        static_cast<__nv_bfloat16*>(out), out_row_stride, rows, cols);
  else
    silu_mul_kernel<__half><<<blocks, threads, 0, st>>>(static_cast<const __half*>(gate),
                                                        static_cast<const __half*>(up), in_row_stride,
                                                        static_cast<__half*>(out), out_row_stride, rows, cols);
  return check_launch();
}

}  // extern "C"
