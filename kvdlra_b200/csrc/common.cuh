// Shared device helpers for the kvdlra_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "kvdlra_b200.h"

#define KVD_DEVICE __device__ __forceinline__

namespace kvd {

// Status words written by kernels instead of trapping (read by kvd_check_status).
enum StatusSlot { kStatusNumeric = 0, kStatusBounds = 1, kStatusTimeout = 2, kStatusAux = 3 };

// ------------------------------------------------------------ dtype I/O

template <typename T> struct IO;
template <> struct IO<float> {
  static KVD_DEVICE float load(const float* p) { return *p; }
  static KVD_DEVICE void store(float* p, float v) { *p = v; }
};
template <> struct IO<__nv_bfloat16> {
  static KVD_DEVICE float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  static KVD_DEVICE void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
};

template <typename T> KVD_DEVICE float load_f(const T* p) { return IO<T>::load(p); }
template <typename T> KVD_DEVICE void store_f(T* p, float v) { IO<T>::store(p, v); }

// ------------------------------------------------------------ ranking

// Total-order key of a score for rank counting: a larger value gets a larger
// key, -0 and +0 tie, and every NaN ties with every other NaN above +inf --
// the order torch's stable sort gives (bug_cache.py:810 argsorts the scores
// with it).  Counting ranks over keys is a strict order with the index as tie
// break, so exactly k candidates have rank < k whatever the inputs hold.
KVD_DEVICE unsigned order_key(float v) {
  unsigned b = __float_as_uint(v);
  if (v != v) b = 0x7fc00000u;
  else if (v == 0.f) b = 0u;
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// ------------------------------------------------------------ reductions

KVD_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
KVD_DEVICE double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
KVD_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------------ RoPE
// The rotary angle of frequency j at position pos, as the model's rotary
// module forms it: one fp32 product pos * inv_freq[j] (exact rounding), then
// cos/sin scaled by attention_scaling.  Full-precision sincosf (no fast math).
KVD_DEVICE void rope_cs(int pos, float inv_freq_j, float scale, float* c, float* s) {
  const float ang = __fmul_rn((float)pos, inv_freq_j);
  float sn, cs;
  sincosf(ang, &sn, &cs);
  *c = __fmul_rn(cs, scale);
  *s = __fmul_rn(sn, scale);
}

// The same cos/sin with the angle reduced by Cody-Waite (argument reduction
// by 2*pi held as three fp32 parts, the first with 8 significant bits so
// k * part1 is exact for |k| < 2^16) and the hardware sin/cos
// approximations on the reduced angle |r| <= pi (absolute error about
// 2^-21): within 1e-6 of rope_cs for |pos * inv_freq| up to ~1e5, at a
// fraction of the instructions.  For kernels that evaluate one angle per
// (token, frequency) in an inner loop.
KVD_DEVICE void rope_cs_fast(int pos, float inv_freq_j, float scale, float* c, float* s) {
  constexpr float kTwoPi1 = 6.28125f;                 // 201 / 32
  constexpr float kTwoPi2 = 1.9353071795864769e-3f;   // 2*pi - kTwoPi1, rounded
  constexpr float kTwoPi3 = 1.0253376606e-11f;         // 2*pi - kTwoPi1 - kTwoPi2, rounded
  constexpr float kInvTwoPi = 0.15915494309189535f;
  const float ang = __fmul_rn((float)pos, inv_freq_j);
  const float k = rintf(ang * kInvTwoPi);
  float r = fmaf(-k, kTwoPi1, ang);
  r = fmaf(-k, kTwoPi2, r);
  r = fmaf(-k, kTwoPi3, r);
  float sn, cs;
  __sincosf(r, &sn, &cs);
  *c = __fmul_rn(cs, scale);
  *s = __fmul_rn(sn, scale);
}

// ------------------------------------------------------------ TF32 MMA
// One warp-level m16n8k8 TF32 product with fp32 accumulation (row-major A,
// column-major B).  Fragments (g = lane / 4, t = lane % 4):
//   A: a0 (g, t), a1 (g + 8, t), a2 (g, t + 4), a3 (g + 8, t + 4)
//   B: b0 (k = t, n = g), b1 (k = t + 4, n = g)
//   C: c0 (g, 2t), c1 (g, 2t + 1), c2 (g + 8, 2t), c3 (g + 8, 2t + 1)
KVD_DEVICE uint32_t tf32_bits(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
KVD_DEVICE void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// x = hi + lo with both parts TF32: three products hi*hi + hi*lo + lo*hi
// carry about 21 significant bits (the "3xTF32" split).
KVD_DEVICE void tf32_split(float x, uint32_t* hi, uint32_t* lo) {
  *hi = tf32_bits(x);
  *lo = tf32_bits(x - __uint_as_float(*hi));
}
// d += A B with A, B given as fp32 fragments; SPLIT = the 3xTF32 product.
template <bool SPLIT>
KVD_DEVICE void mma_f32(float (&d)[4], const float (&a)[4], float b0, float b1) {
  if constexpr (SPLIT) {
    uint32_t ah[4], al[4], bh0, bl0, bh1, bl1;
#pragma unroll
    for (int i = 0; i < 4; ++i) tf32_split(a[i], &ah[i], &al[i]);
    tf32_split(b0, &bh0, &bl0);
    tf32_split(b1, &bh1, &bl1);
    mma_tf32(d, al, bh0, bh1);
    mma_tf32(d, ah, bl0, bl1);
    mma_tf32(d, ah, bh0, bh1);
  } else {
    const uint32_t ah[4] = {tf32_bits(a[0]), tf32_bits(a[1]), tf32_bits(a[2]), tf32_bits(a[3])};
    mma_tf32(d, ah, tf32_bits(b0), tf32_bits(b1));
  }
}

// One warp-level fp64 m8n8k4 product, d += a b (row-major A, column-major B;
// g = lane / 4, t = lane % 4): a = A[g][t], b = B[t][g], d0/d1 = D[g][2t], D[g][2t + 1].
KVD_DEVICE void dmma_8x8x4(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};\n"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}

// Inverse rotation of one rotate-half pair (x1 = x[j], x2 = x[j + D/2]):
// (x cos - rotate_half(x) sin) / scale^2 with rotate_half(x) = [-x2, x1].
KVD_DEVICE void rope_unapply_pair(float x1, float x2, float c, float s, float inv_scale_sq,
                                  float* y1, float* y2) {
  *y1 = (x1 * c + x2 * s) * inv_scale_sq;
  *y2 = (x2 * c - x1 * s) * inv_scale_sq;
}
// Forward rotation: x cos + rotate_half(x) sin.
KVD_DEVICE void rope_apply_pair(float x1, float x2, float c, float s, float* y1, float* y2) {
  *y1 = x1 * c - x2 * s;
  *y2 = x2 * c + x1 * s;
}

KVD_DEVICE int imin(int a, int b) { return a < b ? a : b; }
KVD_DEVICE int imax(int a, int b) { return a > b ? a : b; }

}  // namespace kvd

// Host-side error plumbing shared by the translation units.
namespace kvd_host {
void set_error(const char* fmt, ...);
int check_launch(const char* what);
}  // namespace kvd_host
