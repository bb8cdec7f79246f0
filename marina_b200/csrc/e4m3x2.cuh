// Two-term e4m3 activations (the fp8x2 precision): a value v is carried as hi = e4m3(v) and
// lo = e4m3(v - hi), both with the operand's static scale, and a GEMM runs each MMA step twice (on
// the hi and on the lo codes, against the same e4m3 weights) into one f32 accumulator, which
// therefore sees hi + lo: about twice e4m3's 4 significant bits per activation.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace mrn {

// Two values as two-term e4m3 pairs: hi = e4m3(v) (round to nearest, saturating), lo = e4m3(v -
// hi) with the difference taken exactly in f32 (hi is exact in f16); hi + lo carries about twice
// e4m3's 4 significant bits. Returns the two hi codes and the two lo codes, packed.
__device__ __forceinline__ void split_e4m3x2(float2 v, uint16_t& hi, uint16_t& lo) {
  const __nv_fp8x2_storage_t h = __nv_cvt_float2_to_fp8x2(v, __NV_SATFINITE, __NV_E4M3);
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(h, __NV_E4M3);
  const float2 hf = __half22float2(*reinterpret_cast<const __half2*>(&hr));
  const __nv_fp8x2_storage_t l = __nv_cvt_float2_to_fp8x2(make_float2(v.x - hf.x, v.y - hf.y), __NV_SATFINITE,
                                                          __NV_E4M3);
  hi = h;
  lo = l;
}

// Four values (a.x, a.y, b.x, b.y) as two-term e4m3: the four hi codes and the four lo codes, each
// packed into a word in that order (lowest byte first).
__device__ __forceinline__ void split_e4m3x4(float2 a, float2 b, uint32_t& hi, uint32_t& lo) {
  uint16_t ha, la, hb, lb;
  split_e4m3x2(a, ha, la);
  split_e4m3x2(b, hb, lb);
  hi = static_cast<uint32_t>(ha) | (static_cast<uint32_t>(hb) << 16);
  lo = static_cast<uint32_t>(la) | (static_cast<uint32_t>(lb) << 16);
}

}  // namespace mrn
