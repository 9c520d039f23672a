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
