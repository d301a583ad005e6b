// Rotary embedding of q and k plus the KV-cache append of the rotated k and v,
// in one launch: the step before the verify attention in
// LlamaAttention.forward (llama_target_model.py:765-783: rotary_emb +
// apply_rotary_pos_emb, then past_key_value[0/1].cat, cache_state.py:52-66).
//
// One CTA per (token, batch row).  A thread takes VEC consecutive pairs
// (j, j + D/2) of one head row, so every element it writes depends only on
// what it read itself (q may be rotated in place).  Every product and the sum are rounded
// to the element type, as the reference's torch element-wise ops do, which
// makes the result bit-identical given the same cos / sin tables.
#include <algorithm>

#include "common.cuh"
#include "specverify.h"

namespace tv {
namespace {

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f(float x) { return x; }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ float from_f(float x) { return x; }
// round to the element type, carried as float
template <typename T>
__device__ __forceinline__ float rnd(float x) { return to_f<T>(from_f<T>(x)); }

// VEC consecutive elements moved as one 4-, 8- or 16-byte word.
template <int BYTES> struct Word;
template <> struct Word<4> { using type = uint32_t; };
template <> struct Word<8> { using type = uint2; };
template <> struct Word<16> { using type = uint4; };

template <typename T, int VEC>
__device__ __forceinline__ void loadv(const T* p, float (&f)[VEC]) {
  using W = typename Word<sizeof(T) * VEC>::type;
  const W w = *reinterpret_cast<const W*>(p);
  const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
  for (int i = 0; i < VEC; ++i) f[i] = to_f<T>(e[i]);
}
template <typename T, int VEC>
__device__ __forceinline__ void storev(T* p, const float (&f)[VEC]) {
  using W = typename Word<sizeof(T) * VEC>::type;
  W w;
  T* e = reinterpret_cast<T*>(&w);
#pragma unroll
  for (int i = 0; i < VEC; ++i) e[i] = from_f<T>(f[i]);
  *reinterpret_cast<W*>(p) = w;
}

// R(R(x c) + R(r s)) with products of 16-bit values exact in fp32 and, for
// fp32, no contraction into a fused multiply-add.
template <typename T>
__device__ __forceinline__ float rope1(float x, float c, float r, float s) {
  return rnd<T>(__fadd_rn(rnd<T>(__fmul_rn(x, c)), rnd<T>(__fmul_rn(r, s))));
}

// A CTA takes `tok` consecutive tokens of one batch row; work item w is VEC
// consecutive elements j of the first half of one head row of one token and
// the matching VEC of the second half.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) rope_append_kernel(const tv_rope_args a, int tok) {
  const int b = blockIdx.y;
  const int t_base = blockIdx.x * tok;
  const int h2 = a.head_dim / 2;
  const int tpr = h2 / VEC;                          // work items per head row
  const int nq = a.heads, nk = a.kv_heads;
  const bool append = a.k_cache != nullptr;
  const int nv = append && a.v ? a.kv_heads : 0;
  const int per_tok = (nq + nk + nv) * tpr;          // q heads, k heads, v heads
  const int ntok = min(tok, a.tokens - t_base);
  for (int w = threadIdx.x; w < ntok * per_tok; w += blockDim.x) {
    const int ti = w / per_tok;
    const int rem = w - ti * per_tok;
    const int hr = rem / tpr;
    const int j = (rem - hr * tpr) * VEC;
    const int t = t_base + ti;
    const int64_t row = a.pos ? a.pos[(int64_t)b * a.pos_sb + t] : (int64_t)t;
    const int64_t idx = a.start + t;                 // token index in the cache
    bool ok = row >= 0 && row < a.cs_rows;
    int64_t kc_off = 0, vc_off = 0;
    if (append) {
      if (a.page_table) {
        const int32_t pg = idx >= 0 ? a.page_table[(int64_t)b * a.pt_sb + idx / a.page_size] : -1;
        const int slot = (int)(idx % a.page_size);
        if (pg < 0 || pg >= a.num_pages) ok = false;
        kc_off = (int64_t)pg * a.kc_sb + (int64_t)slot * a.kc_st;
        vc_off = (int64_t)pg * a.vc_sb + (int64_t)slot * a.vc_st;
      } else {
        if (idx < 0 || idx >= a.capacity) ok = false;
        kc_off = (int64_t)b * a.kc_sb + idx * a.kc_st;
        vc_off = (int64_t)b * a.vc_sb + idx * a.vc_st;
      }
    }
    if (!ok) {                                       // the whole token is skipped
      if (rem == 0 && a.status) atomicExch(a.status, TV_ERR_INPUT);
      continue;
    }
    float x1[VEC], x2[VEC];
    if (hr >= nq + nk) {                             // v: plain copy into the cache
      const int h = hr - nq - nk;
      const T* src = static_cast<const T*>(a.v) + (int64_t)b * a.v_sb + (int64_t)h * a.v_sh + (int64_t)t * a.v_st;
      T* dst = static_cast<T*>(a.v_cache) + vc_off + (int64_t)h * a.vc_sh;
      loadv<T, VEC>(src + j, x1);
      loadv<T, VEC>(src + j + h2, x2);
      storev<T, VEC>(dst + j, x1);
      storev<T, VEC>(dst + j + h2, x2);
      continue;
    }
    const T* cs = static_cast<const T*>(a.cos) + (int64_t)b * a.cs_sb + row * a.cs_sr;
    const T* sn = static_cast<const T*>(a.sin) + (int64_t)b * a.cs_sb + row * a.cs_sr;
    const bool is_q = hr < nq;
    const int h = is_q ? hr : hr - nq;
    const T* src = is_q ? static_cast<const T*>(a.q) + (int64_t)b * a.q_sb + (int64_t)h * a.q_sh + (int64_t)t * a.q_st
                        : static_cast<const T*>(a.k) + (int64_t)b * a.k_sb + (int64_t)h * a.k_sh + (int64_t)t * a.k_st;
    float c1[VEC], c2[VEC], s1[VEC], s2[VEC], o1[VEC], o2[VEC];
    loadv<T, VEC>(src + j, x1);
    loadv<T, VEC>(src + j + h2, x2);
    loadv<T, VEC>(cs + j, c1);
    loadv<T, VEC>(cs + j + h2, c2);
    loadv<T, VEC>(sn + j, s1);
    loadv<T, VEC>(sn + j + h2, s2);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      // rotate_half: the first half takes -x2, the second half x1
      o1[i] = rope1<T>(x1[i], c1[i], -x2[i], s1[i]);
      o2[i] = rope1<T>(x2[i], c2[i], x1[i], s2[i]);
    }
    if (is_q) {
      T* dst = static_cast<T*>(a.q_out) + (int64_t)b * a.qo_sb + (int64_t)h * a.qo_sh + (int64_t)t * a.qo_st;
      storev<T, VEC>(dst + j, o1);
      storev<T, VEC>(dst + j + h2, o2);
    } else {
      if (a.k_out) {
        T* dst = static_cast<T*>(a.k_out) + (int64_t)b * a.ko_sb + (int64_t)h * a.ko_sh + (int64_t)t * a.ko_st;
        storev<T, VEC>(dst + j, o1);
        storev<T, VEC>(dst + j + h2, o2);
      }
      if (append) {
        T* dst = static_cast<T*>(a.k_cache) + kc_off + (int64_t)h * a.kc_sh;
        storev<T, VEC>(dst + j, o1);
        storev<T, VEC>(dst + j + h2, o2);
      }
    }
  }
}

}  // namespace
}  // namespace tv

using namespace tv;

extern "C" int tv_rope_append(const tv_rope_args* a, void* stream) {
  if (!a) return TV_ERR_NULL;
  if (a->batch < 0 || a->tokens < 0 || a->heads < 1 || a->kv_heads < 1) return TV_ERR_SHAPE;
  if (a->batch == 0 || a->tokens == 0) return TV_OK;   // nothing to do (empty tensors carry no pointer)
  if (!a->q || !a->k || !a->cos || !a->sin || !a->q_out) return TV_ERR_NULL;
  if (a->head_dim < 4 || a->head_dim > 256 || (a->head_dim % 4) != 0) return TV_ERR_SHAPE;
  if (a->cs_rows < 1) return TV_ERR_SHAPE;
  if (a->k_cache && (!a->v_cache || !a->v)) return TV_ERR_NULL;
  if (a->k_cache && a->page_table && (a->page_size < 1 || a->num_pages < 1)) return TV_ERR_SHAPE;
  if (a->dtype != TV_BF16 && a->dtype != TV_F16 && a->dtype != TV_F32) return TV_ERR_DTYPE;
  // Elements move in words of VEC: 16 bytes where every pointer, stride and
  // half-row allows it, else pairs (4 or 8 bytes).
  const int64_t es = a->dtype == TV_F32 ? 4 : 2;
  const int64_t strides[] = {a->q_sb, a->q_sh, a->q_st, a->k_sb, a->k_sh, a->k_st, a->v_sb, a->v_sh, a->v_st,
                             a->cs_sb, a->cs_sr, a->qo_sb, a->qo_sh, a->qo_st, a->ko_sb, a->ko_sh, a->ko_st,
                             a->kc_sb, a->kc_sh, a->kc_st, a->vc_sb, a->vc_sh, a->vc_st};
  const void* ptrs[] = {a->q, a->k, a->v, a->cos, a->sin, a->q_out, a->k_out, a->k_cache, a->v_cache};
  auto fits = [&](int64_t vec) {
    if ((a->head_dim / 2) % vec) return false;
    for (int64_t s : strides)
      if (s % vec) return false;
    for (const void* p : ptrs)
      if (p && (reinterpret_cast<uintptr_t>(p) % (vec * es))) return false;
    return true;
  };
  const int64_t wide = 16 / es;
  const int vec = fits(wide) ? (int)wide : (fits(2) ? 2 : 0);
  if (!vec) return TV_ERR_ALIGN;
  if (a->batch > 65535) return TV_ERR_SHAPE;
  // Several tokens per CTA (up to about eight work items per thread: loads
  // in flight, fewer CTAs to launch) only once there are more than eight
  // CTAs per SM to share.
  const int64_t per_tok = (int64_t)(a->heads + 2 * a->kv_heads) * (a->head_dim / 2 / vec);
  const int64_t fill = (int64_t)a->tokens * a->batch / (8 * kNumSMs);
  const int tok = (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(64, 2048 / per_tok), fill));
  const dim3 grid((unsigned)((a->tokens + tok - 1) / tok), (unsigned)a->batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->dtype == TV_BF16) {
    if (vec == 8) rope_append_kernel<__nv_bfloat16, 8><<<grid, 256, 0, st>>>(*a, tok);
    else rope_append_kernel<__nv_bfloat16, 2><<<grid, 256, 0, st>>>(*a, tok);
  } else if (a->dtype == TV_F16) {
    if (vec == 8) rope_append_kernel<__half, 8><<<grid, 256, 0, st>>>(*a, tok);
    else rope_append_kernel<__half, 2><<<grid, 256, 0, st>>>(*a, tok);
  } else {
    if (vec == 4) rope_append_kernel<float, 4><<<grid, 256, 0, st>>>(*a, tok);
    else rope_append_kernel<float, 2><<<grid, 256, 0, st>>>(*a, tok);
  }
  return check_launch();
}
