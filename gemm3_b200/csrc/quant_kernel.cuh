// NVFP4 quantiser, dequantiser, scale swizzle and tensor amax for sm_100a.
//
// The quantiser reproduces nvfp4_gemm_cute/quant.py:41-59 bit for bit:
//   xb    = float(x) * gs                                   (one FP32 multiply)
//   amax  = max |xb| over 16 consecutive K elements         (NaN propagates, like torch.amax)
//   scale = e4m3fn(amax / 6)  round-to-nearest-even, overflow -> NaN (no saturation)
//   q     = scale > 0 ? xb / scale : 0                      (IEEE division)
//   code  = argmin_i (|min(|q|, 6) - E2M1[i]| + (i odd) * 1e-6f), first index on ties
//           | 8 if q < 0                                     (quant.py:15-28)
// The code is a monotone step function of |q|: the reference's FP32 distances to the two
// bracketing table entries move in opposite directions as |q| grows, and every other entry is at
// least 0.5 further away. So code = the number of thresholds T1..T7 that |q| reaches, where Tk is
// the smallest float that the reference rounds to code k (found by bisection with the CPU
// restatement and checked against it for every float in [0, 6]; |q| >= 6 clamps to code 7).
//
// q itself is the IEEE quotient xb / scale. A scale is an E4M3 value, so its significand is one
// of eight values 1 + m/8. With r = the correctly rounded 1/scale (one reciprocal per block),
// Markstein's correction  q1 = xb*r, rem = fma(-q1, scale, xb), q = fma(rem, r, q1)  returns
// the correctly rounded quotient for all 2^23 significands of xb and all eight of the scale
// (checked exhaustively on the CPU); exponents only shift the result while no intermediate
// leaves the normal range, which holds for |xb| >= 2^-100. Below that |q| < 2^-91, so the
// magnitude code is 0 however q rounds, and the sign bit is decided from xb and the scale
// directly (e2m1_pack16). Blocks whose every |xb| is at least 2^-100 (the common case) take
// e2m1_pack8_fast, which converts x * (gs / d) slightly scaled down and up, and forms the exact
// quotient only for the rare element that lies next to a rounding tie.
//
// The codes themselves come from the hardware E2M1 conversion (round-to-nearest-even); the
// reference's tie rule is applied exactly by a check that sends only elements next to a rounding
// tie to its thresholds. The block scale goes through the hardware E4M3 conversion, with the
// reference's overflow to NaN applied by one compare (e4m3_encode_nonneg).
//
// For 16-bit inputs whose rows hold whole pairs of blocks one thread owns two neighbouring
// 16-element blocks (nvfp4_quantize_pair_kernel); otherwise one (nvfp4_quantize_kernel).
// Consecutive threads own consecutive blocks of the row-major input, so loads (32 or 64 bytes
// per thread), code stores (8 or 16 bytes) and linear scale stores are coalesced; the swizzled
// scales go to their 128x4-tile position.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "ptx.cuh"

namespace g3 {

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t sign = (b & 0x80u) << 24;
  const uint32_t e = (b >> 3) & 0xFu;
  const uint32_t m = b & 7u;
  if (e == 0xFu && m == 7u) return __uint_as_float(sign | 0x7FC00000u);
  if (e == 0) return __uint_as_float(sign | __float_as_uint(static_cast<float>(m) * 0.001953125f));
  return __uint_as_float(sign | ((e + 120u) << 23) | (m << 20));
}

// FP32 -> E4M3 (fn variant: bias 7, max 448, 0x7F/0xFF = NaN, no infinities) as torch's
// float8_e4m3fn cast does it: round to nearest even, non-saturating. cvt.rn.satfinite.e4m3x2.f32
// rounds the same way but saturates, so anything above 464 (the midpoint between 448 and the
// first value past it, which ties down to 448) and NaN are mapped to 0x7F by one compare; s is
// never negative here. E4M3 values are exact in FP16, so the decode goes through
// cvt.rn.f16x2.e4m3x2 (e4m3_to_f32 below is the bit-level decode the dequantiser uses).
__device__ __forceinline__ uint32_t e4m3_encode_nonneg(float s) {
  uint16_t h;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(h) : "f"(0.0f), "f"(s));
  return s <= 464.0f ? static_cast<uint32_t>(h & 0xFFu) : 0x7Fu;
}

__device__ __forceinline__ float e4m3_decode(uint32_t b) {
  uint32_t h2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(static_cast<uint16_t>(b)));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
}

__device__ __constant__ float kE2M1Table[9] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f, 6.0f};

// Smallest FP32 |q| (as bits) that the reference rounds to E2M1 codes 1..7 (quant.py:15-28): the
// midpoints 0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5 moved by the 1e-6 penalty on odd codes.
constexpr uint32_t kE2M1T1 = 0x3E800012u, kE2M1T2 = 0x3F3FFFF8u, kE2M1T3 = 0x3FA00005u, kE2M1T4 = 0x3FDFFFFCu,
                   kE2M1T5 = 0x40200003u, kE2M1T6 = 0x405FFFFEu, kE2M1T7 = 0x40A00002u;

// kE2M1Next[c]: the reference's threshold (as bits) for rounding to code c + 1, +inf past code 7.
__device__ __constant__ uint32_t kE2M1Next[8] = {kE2M1T1, kE2M1T2, kE2M1T3, kE2M1T4,
                                                 kE2M1T5, kE2M1T6, kE2M1T7, 0x7F800000u};

// Exact E2M1 magnitude code of |q| = mag by the reference's thresholds, given c = the
// round-to-nearest-even code of mag * (1 - 2^-17) where that of mag * (1 + 2^-17) is c + 1: the
// two conversions bracket the one rounding tie next to mag, and the reference moves each tie by
// at most 18 ulps, so its code is c or c + 1, decided by one exact float comparison with the
// threshold of code c + 1.
__device__ __forceinline__ uint32_t e2m1_mag_code_near_tie(float mag, uint32_t c) {
  return c + (mag >= __uint_as_float(kE2M1Next[c & 7u]) ? 1u : 0u);
}

// Hardware round-to-nearest-even of eight magnitudes to E2M1 (saturating at 6), packed two per
// byte with element 2i in the low nibble: four cvt.e2m1x2 into one word.
__device__ __forceinline__ uint32_t cvt_e2m1x8(const float (&m)[8]) {
  uint32_t w;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(w)
      : "f"(m[0]), "f"(m[1]), "f"(m[2]), "f"(m[3]), "f"(m[4]), "f"(m[5]), "f"(m[6]), "f"(m[7]));
  return w;
}

// Packed E2M1 codes (sign in bit 3, element 2i in the low nibble) of the eight quotients
// xb[i] / d, given r = the correctly rounded 1 / d and d_lo = d * 2^-50.
//  - magnitude: the reference's code equals round-to-nearest-even on the E2M1 grid except for
//    |q| within a few ulps of one of the seven rounding ties, where its 1e-6 bias on odd codes
//    moves the boundary (within 18 ulps, relative 2.2e-6). The hardware conversions of
//    |q| * (1 - 2^-17) and |q| * (1 + 2^-17) agree exactly when no tie lies in between, and
//    then that code is the reference's (checked on the CPU for every float in [0, 6.5]). An
//    element whose two conversions differ gets the exact code from the one threshold between
//    them (e2m1_mag_code_near_tie).
//  - sign: q = RN(xb / d) < 0 exactly when xb / d < -2^-150 (the tie at 2^-150 rounds to -0),
//    i.e. when t = -xb * 2^100 - d * 2^-50 > 0; both products are exact and the FMA keeps the
//    sign, so the bit is t's "greater than +0" test on its bit pattern (t is never -0: d > 0).
//    Tiny xb therefore needs no division: its magnitude code is 0 whatever rounding the quotient
//    sees, and its sign comes from xb and d directly.
__device__ __forceinline__ uint32_t e2m1_pack8(const float* xb, float d, float r, float d_lo) {
  float mag[8], lo[8], hi[8];
  uint32_t neg = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float q1 = __fmul_rn(xb[i], r);
    const float rem = __fmaf_rn(q1, -d, xb[i]);
    mag[i] = fabsf(__fmaf_rn(rem, r, q1));
    lo[i] = __fmul_rn(mag[i], 0x1.ffffp-1f);   // 1 - 2^-17
    hi[i] = __fmul_rn(mag[i], 0x1.00008p+0f);  // 1 + 2^-17
    const float t = __fmaf_rn(-xb[i], 0x1p100f, -d_lo);
    neg |= ((0u - __float_as_uint(t)) >> 31) << (4 * i + 3);
  }
  uint32_t w = cvt_e2m1x8(lo);
  const uint32_t near_tie = w ^ cvt_e2m1x8(hi);
  if (near_tie != 0u) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((near_tie >> (4 * i)) & 0xFu)
        w = (w & ~(0xFu << (4 * i))) | (e2m1_mag_code_near_tie(mag[i], (w >> (4 * i)) & 0x7u) << (4 * i));
  }
  return w | neg;
}

__device__ __forceinline__ uint2 e2m1_pack16(const float (&xb)[16], float d, float r) {
  const float d_lo = __fmul_rn(d, 0x1p-50f);
  return make_uint2(e2m1_pack8(xb, d, r, d_lo), e2m1_pack8(xb + 8, d, r, d_lo));
}

// Approximate reciprocal (MUFU; at most a couple of ulps from 1/d, d a normal float).
__device__ __forceinline__ float rcp_approx(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}

// Packed E2M1 codes of eight elements of a block whose every |xb| = |x * gs| is at least 2^-100,
// from the raw inputs x: one paired multiply per two elements and side.
//  - For such a block q = RN(xb / d) is a nonzero normal float with the sign of xb, so the
//    reference's sign test q < 0 is the sign of x * gs, which the conversions set themselves (a
//    negative q whose magnitude rounds to 0 gives code 8, as in the reference).
//  - lo = x * RN(RN(gs * ~1/d) * (1 - 2^-17)) and hi likewise with (1 + 2^-17) are within a few
//    ulps (relative 6e-7) of q * (1 -+ 2^-17), while the reference's rounding rule differs from
//    round-to-nearest-even only within 2.2e-6 of a tie. So where the hardware conversions of lo
//    and hi agree, no tie lies within 5e-6 of q and that code is the reference's.
//  - An element whose two conversions differ takes the exact path: xb = RN(x * gs), the
//    correctly rounded quotient by Markstein's correction with r = RN(1 / d), and the one
//    threshold between the two codes. Only the magnitude bits are replaced; lo and hi carry the
//    same sign.
__device__ __forceinline__ uint32_t e2m1_pack8_fast(const float* x, float gs, float d, float clo, float chi) {
  const float2 clo2 = make_float2(clo, clo), chi2 = make_float2(chi, chi);
  float lo[8], hi[8];
#pragma unroll
  for (int i = 0; i < 8; i += 2) {
    const float2 xx = make_float2(x[i], x[i + 1]);
    const float2 l = __fmul2_rn(xx, clo2), h = __fmul2_rn(xx, chi2);
    lo[i] = l.x;
    lo[i + 1] = l.y;
    hi[i] = h.x;
    hi[i + 1] = h.y;
  }
  uint32_t w = cvt_e2m1x8(lo);
  const uint32_t near_tie = w ^ cvt_e2m1x8(hi);
  if (near_tie != 0u) {
    const float r = __frcp_rn(d);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if ((near_tie >> (4 * i)) & 0xFu) {
        const float xb = __fmul_rn(x[i], gs);
        const float q1 = __fmul_rn(xb, r);
        const float rem = __fmaf_rn(q1, -d, xb);
        const float q = __fmaf_rn(rem, r, q1);
        w = (w & ~(0x7u << (4 * i))) | (e2m1_mag_code_near_tie(fabsf(q), (w >> (4 * i)) & 0x7u) << (4 * i));
      }
  }
  return w;
}

// max(a, b, c), NaN if any of them is NaN; min(a, b, c) ignoring NaN (sm_100 three-input forms).
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float min3(float a, float b, float c) {
  float d;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Byte offset of scale (row, col) in the 128x4 swizzled layout with `c4` 4-column groups.
__device__ __forceinline__ int64_t sf_swizzle_offset(int64_t row, int64_t col, int64_t c4) {
  return ((row >> 7) * c4 + (col >> 2)) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (col & 3);
}

// The raw bits of one 16-element block: 32 bytes of f16/bf16 or 64 bytes of f32.
template <int kInDtype>  // 0 = f16, 1 = bf16, 2 = f32
struct RawBlock {
  uint4 w[kInDtype == 2 ? 4 : 2];
};

template <int kInDtype>
__device__ __forceinline__ void load_raw(const void* base, int64_t elem, RawBlock<kInDtype>& rb) {
  const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(base) + elem * (kInDtype == 2 ? 4 : 2));
#pragma unroll
  for (int i = 0; i < (kInDtype == 2 ? 4 : 2); ++i) rb.w[i] = __ldg(p + i);
}

template <int kInDtype>
__device__ __forceinline__ void unpack_raw(const RawBlock<kInDtype>& rb, float (&v)[16]) {
#pragma unroll
  for (int i = 0; i < (kInDtype == 2 ? 4 : 2); ++i) {
    const uint32_t ws[4] = {rb.w[i].x, rb.w[i].y, rb.w[i].z, rb.w[i].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (kInDtype == 2) {
        v[4 * i + j] = __uint_as_float(ws[j]);
      } else {
        // x + (-0) with a 16-bit operand and an FP32 result (sm_100's mixed-precision add): exact,
        // keeps the sign of zero, and runs on the FMA pipe where shifts and masks would take the
        // ALU pipe, the kernel's busiest (8192^2 BF16: ALU instructions -11 %, 35.3 -> 34.9 us).
        if constexpr (kInDtype == 1)
          asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
              "add.rn.f32.bf16 %0, l, %3;\n\tadd.rn.f32.bf16 %1, h, %3;\n\t}"
              : "=f"(v[8 * i + 2 * j]), "=f"(v[8 * i + 2 * j + 1])
              : "r"(ws[j]), "f"(-0.0f));
        else
          asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\t"
              "add.rn.f32.f16 %0, l, %3;\n\tadd.rn.f32.f16 %1, h, %3;\n\t}"
              : "=f"(v[8 * i + 2 * j]), "=f"(v[8 * i + 2 * j + 1])
              : "r"(ws[j]), "f"(-0.0f));
      }
    }
  }
}

template <int kInDtype>
__device__ __forceinline__ void load16(const void* base, int64_t elem, float (&v)[16]) {
  RawBlock<kInDtype> rb;
  load_raw<kInDtype>(base, elem, rb);
  unpack_raw<kInDtype>(rb, v);
}

struct QuantParams {
  const void* x;
  int64_t rows, k;          // logical shape
  int64_t cols;             // k / 16
  int64_t rows_pad, cols_pad;  // scale grid padded to 128 rows, 4 columns
  float gs;
  const float* gs_dev;
  int gs_mode;
  int div_mode;
  uint8_t* packed;
  uint8_t* sf_swz;
  uint8_t* sf_lin;
  float* gs_out;
};

__device__ __forceinline__ float resolve_global_scale(const QuantParams& p) {
  if (p.gs_mode == 0) return p.gs;
  const float v = *p.gs_dev;
  if (p.gs_mode == 1) return v;
  // gs_mode 2: v is the tensor amax; encode scale 448 * 6 / amax.
  return (v > 0.0f && v <= 3.402823466e38f) ? __fdiv_rn(2688.0f, v) : 1.0f;
}

// The scale byte and packed codes of one 16-element block of input values.
//  - The block amax and smallest magnitude are taken over the raw |x| and scaled once: RN(. * |gs|)
//    is monotone, so RN(max|x| * |gs|) = max |RN(x * gs)| = the reference's amax of xb (NaN and
//    infinities propagate the same way), and likewise for the minimum.
//  - Blocks whose every |xb| is at least 2^-100 (the common case) take e2m1_pack8_fast; blocks
//    holding a zero or a smaller magnitude take the general path, which forms xb and decides
//    signs without the quotient.
template <int kInDtype>
__device__ __forceinline__ uint32_t quantize_values(const RawBlock<kInDtype>& rb, float gs, int div_mode, uint2& codes) {
  const float inv6 = 0.166666672f;  // fl(1/6): what torch on CUDA multiplies by for "/ 6.0"
  float v[16];
  unpack_raw<kInDtype>(rb, v);
  // A NaN element makes amax NaN and an infinite one makes it Inf: the reference's scale is NaN
  // either way (NaN amax, or Inf / 6 overflowing E4M3), and e4m3_encode_nonneg maps both to 0x7F.
  float amax = max3_nan(fabsf(v[0]), fabsf(v[1]), fabsf(v[2]));
  float mn = min3(fabsf(v[0]), fabsf(v[1]), fabsf(v[2]));
#pragma unroll
  for (int i = 3; i < 15; i += 2) {
    amax = max3_nan(amax, fabsf(v[i]), fabsf(v[i + 1]));
    mn = min3(mn, fabsf(v[i]), fabsf(v[i + 1]));
  }
  amax = max_nan(amax, fabsf(v[15]));
  mn = fminf(mn, fabsf(v[15]));
  const float ags = fabsf(gs);
  amax = __fmul_rn(amax, ags);
  mn = __fmul_rn(mn, ags);
  const float s = div_mode == 0 ? __fmul_rn(amax, inv6) : __fdiv_rn(amax, 6.0f);
  const uint32_t sf = e4m3_encode_nonneg(s);
  const float denom = e4m3_decode(sf);
  // else q = 0 for every element: code 0 (a NaN scale included)
  codes = make_uint2(0u, 0u);
  if (denom > 0.0f) {
    // g = gs / d must be a normal float for the products x * g to keep their precision.
    const float g = __fmul_rn(gs, rcp_approx(denom));
    if (mn >= 0x1p-100f && fabsf(g) >= 0x1p-125f && fabsf(g) <= 0x1p+125f) {
      const float clo = __fmul_rn(g, 0x1.ffffp-1f);   // 1 - 2^-17
      const float chi = __fmul_rn(g, 0x1.00008p+0f);  // 1 + 2^-17
      codes = make_uint2(e2m1_pack8_fast(v, gs, denom, clo, chi), e2m1_pack8_fast(v + 8, gs, denom, clo, chi));
    } else {
      const float2 gs2 = make_float2(gs, gs);
#pragma unroll
      for (int i = 0; i < 16; i += 2) {
        const float2 xb = __fmul2_rn(make_float2(v[i], v[i + 1]), gs2);
        v[i] = xb.x;
        v[i + 1] = xb.y;
      }
      codes = e2m1_pack16(v, denom, __frcp_rn(denom));
    }
  }
  return sf;
}

// One 16-element block (r, c) of the padded scale grid: codes, linear and swizzled scale. Blocks
// outside the logical shape write a zero scale into the swizzled padding only.
template <int kInDtype, typename Idx>
__device__ __forceinline__ void quantize_block(const QuantParams& p, float gs, Idx r, Idx c, Idx c4, Idx elem,
                                               bool inside, const RawBlock<kInDtype>& rb) {
  uint32_t sf = 0;
  if (inside) {
    uint2 codes;
    sf = quantize_values<kInDtype>(rb, gs, p.div_mode, codes);
    // elem = r * k + 16 c: the block's codes start at byte elem / 2, its linear scale at elem / 16
    *reinterpret_cast<uint2*>(p.packed + (elem >> 1)) = codes;
    if (p.sf_lin != nullptr) p.sf_lin[elem >> 4] = static_cast<uint8_t>(sf);
  }
  p.sf_swz[((r >> 7) * c4 + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 + (c & 3)] = static_cast<uint8_t>(sf);
}

// The grid-stride walk over the blocks (r, c) of the padded scale grid, advanced by the stride
// without dividing. Idx is uint32_t when every element offset of the padded grid fits in 32 bits
// (the host checks rows_pad * k < 2^32), which keeps the per-block index arithmetic to single
// instructions; int64_t otherwise. Loading the next block before converting the current one
// pays for f32 inputs (8192^2: 50.0 -> 47.0 us) but not for 16-bit ones (no change, 16 more
// registers), which instead run at 32 registers and eight CTAs per SM (43.0 -> 42.3 us).
template <int kInDtype, typename Idx>
__device__ __forceinline__ void quantize_grid_stride(const QuantParams& p, float gs) {
  const Idx rows = static_cast<Idx>(p.rows), cols = static_cast<Idx>(p.cols), k = static_cast<Idx>(p.k);
  const Idx cols_pad = static_cast<Idx>(p.cols_pad);
  const Idx total = static_cast<Idx>(p.rows_pad) * cols_pad;
  const Idx c4 = cols_pad >> 2;
  const Idx stride = static_cast<Idx>(gridDim.x) * blockDim.x;
  const Idx b0 = static_cast<Idx>(blockIdx.x) * blockDim.x + threadIdx.x;
  const Idx dr = stride / cols_pad, dc = stride - dr * cols_pad;
  Idx r = b0 / cols_pad, c = b0 - r * cols_pad;
  if constexpr (kInDtype != 2) {
    for (Idx b = b0; b < total; b += stride) {
      const bool inside = r < rows && c < cols;
      const Idx elem = r * k + c * 16;
      RawBlock<kInDtype> rb;
      if (inside) load_raw<kInDtype>(p.x, static_cast<int64_t>(elem), rb);
      quantize_block<kInDtype, Idx>(p, gs, r, c, c4, elem, inside, rb);
      c += dc;
      r += dr;
      if (c >= cols_pad) {
        c -= cols_pad;
        ++r;
      }
    }
  } else {
    // f32: the next block's 64 bytes are loaded before the current block is converted
    bool next_inside = b0 < total && r < rows && c < cols;
    Idx next_elem = r * k + c * 16;
    RawBlock<kInDtype> next;
    if (next_inside) load_raw<kInDtype>(p.x, static_cast<int64_t>(next_elem), next);
    for (Idx b = b0; b < total; b += stride) {
      const RawBlock<kInDtype> rb = next;
      const bool inside = next_inside;
      const Idx elem = next_elem, cr = r, cc = c;
      c += dc;
      r += dr;
      if (c >= cols_pad) {
        c -= cols_pad;
        ++r;
      }
      next_inside = b + stride < total && r < rows && c < cols;
      next_elem = r * k + c * 16;
      if (next_inside) load_raw<kInDtype>(p.x, static_cast<int64_t>(next_elem), next);
      quantize_block<kInDtype, Idx>(p, gs, cr, cc, c4, elem, inside, rb);
    }
  }
}

template <int kInDtype, typename Idx>
__global__ void __launch_bounds__(256, kInDtype == 2 ? 4 : (sizeof(Idx) == 4 ? 8 : 5)) nvfp4_quantize_kernel(const QuantParams p) {
  const float gs = resolve_global_scale(p);
  if (p.gs_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *p.gs_out = gs;
  quantize_grid_stride<kInDtype, Idx>(p, gs);
}

// Two consecutive blocks of a row per thread, for 16-bit inputs: 64 bytes loaded per thread (as
// one f32 block), one 16-byte code store and one 16-bit store of the two scales in each layout.
// The host takes it when k % 32 == 0 (so both blocks of a pair are inside the row or both in the
// padding), rows_pad * k < 2^32, the packed codes are 16-byte and both scale arrays 2-byte
// aligned. The per-element arithmetic is nvfp4_quantize_kernel's.
template <int kInDtype>
__global__ void __launch_bounds__(256) nvfp4_quantize_pair_kernel(const QuantParams p) {
  static_assert(kInDtype != 2, "f32 inputs use nvfp4_quantize_kernel");
  const float gs = resolve_global_scale(p);
  if (p.gs_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *p.gs_out = gs;
  const uint32_t rows = static_cast<uint32_t>(p.rows), cols = static_cast<uint32_t>(p.cols);
  const uint32_t k = static_cast<uint32_t>(p.k);
  const uint32_t c2 = static_cast<uint32_t>(p.cols_pad >> 1);  // block pairs per padded row
  const uint32_t c4 = static_cast<uint32_t>(p.cols_pad >> 2);
  const uint32_t total = static_cast<uint32_t>(p.rows_pad) * c2;
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t b0 = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t dr = stride / c2, dq = stride - dr * c2;
  uint32_t r = b0 / c2, q = b0 - r * c2;
  for (uint32_t b = b0; b < total; b += stride) {
    const uint32_t c = 2 * q;
    uint32_t sf2 = 0;
    if (r < rows && c < cols) {
      const uint32_t elem = r * k + c * 16;
      RawBlock<kInDtype> rb0, rb1;
      load_raw<kInDtype>(p.x, static_cast<int64_t>(elem), rb0);
      load_raw<kInDtype>(p.x, static_cast<int64_t>(elem + 16), rb1);
      uint2 w0, w1;
      sf2 = quantize_values<kInDtype>(rb0, gs, p.div_mode, w0);
      sf2 |= quantize_values<kInDtype>(rb1, gs, p.div_mode, w1) << 8;
      *reinterpret_cast<uint4*>(p.packed + (elem >> 1)) = make_uint4(w0.x, w0.y, w1.x, w1.y);
      if (p.sf_lin != nullptr) *reinterpret_cast<uint16_t*>(p.sf_lin + (elem >> 4)) = static_cast<uint16_t>(sf2);
    }
    *reinterpret_cast<uint16_t*>(p.sf_swz + ((r >> 7) * c4 + (c >> 2)) * 512 + (r & 31) * 16 + ((r & 127) >> 5) * 4 +
                                 (c & 3)) = static_cast<uint16_t>(sf2);
    q += dq;
    r += dr;
    if (q >= c2) {
      q -= c2;
      ++r;
    }
  }
}

// Activation quantiser for an LLM projection call, as two launches chained by programmatic
// dependent launch (each lets the next kernel in the stream start as its first instruction):
//   nvfp4_act_amax_kernel      every CTA writes the max |x| bits of its grid-stride share to
//                              parts[blockIdx.x] (no atomics, so nothing needs zeroing first);
//   nvfp4_act_quantize_kernel  waits for the amax kernel, reduces the partial maxima in every CTA,
//                              derives gs = 2688 / amax with the same rule as gs_mode 2 and, in
//                              CTA 0, writes gs and the GEMM alpha 1 / (gs * gs_other); then the
//                              grid-stride quantisation of nvfp4_quantize_kernel.
// A weight-streaming GEMM launched after them with programmatic dependent launch starts reading
// its weights while these run.
constexpr int kActThreads = 256;
constexpr int kActMaxParts = 1024;

template <int kInDtype>
__global__ void __launch_bounds__(kActThreads) nvfp4_act_amax_kernel(const void* x, int64_t numel, uint32_t* parts) {
  __shared__ uint32_t warp_max[kActThreads / 32];
  griddep_launch_dependents();
  uint32_t m = 0;
  const int64_t nvec = numel >> 4;  // numel is a multiple of 16
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * kActThreads + threadIdx.x; b < nvec;
       b += static_cast<int64_t>(gridDim.x) * kActThreads) {
    float v[16];
    load16<kInDtype>(x, b * 16, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = max(m, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t w = threadIdx.x < kActThreads / 32 ? warp_max[threadIdx.x] : 0u;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = max(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) parts[blockIdx.x] = w;
  }
}

template <int kInDtype, typename Idx>
__global__ void __launch_bounds__(kActThreads)
    nvfp4_act_quantize_kernel(const QuantParams p, const uint32_t* parts, int n_parts, const float* gs_other,
                              float* alpha_out) {
  __shared__ uint32_t warp_max[kActThreads / 32];
  griddep_launch_dependents();
  griddep_wait();  // the amax kernel has finished and its parts are visible
  uint32_t m = 0;
  for (int i = threadIdx.x; i < n_parts; i += kActThreads) m = max(m, parts[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  uint32_t bits = 0;
#pragma unroll
  for (int w = 0; w < kActThreads / 32; ++w) bits = max(bits, warp_max[w]);
  const float amax = __uint_as_float(bits);
  const float gs = (amax > 0.0f && amax <= 3.402823466e38f) ? __fdiv_rn(2688.0f, amax) : 1.0f;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    if (p.gs_out != nullptr) *p.gs_out = gs;
    if (alpha_out != nullptr) *alpha_out = __frcp_rn(__fmul_rn(gs, *gs_other));
  }
  quantize_grid_stride<kInDtype, Idx>(p, gs);
}

struct DequantParams {
  const uint8_t* packed;
  const uint8_t* sf_lin;
  int64_t rows, k, cols;
  float gs;
  int div_mode;
  float* out;
};

__global__ void __launch_bounds__(256) nvfp4_dequantize_kernel(const DequantParams p) {
  const int64_t total = p.rows * p.cols;
  const float inv_gs = __fdiv_rn(1.0f, p.gs);
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = b / p.cols;
    const int64_t c = b - r * p.cols;
    const float scale = e4m3_to_f32(p.sf_lin[b]);
    const uint2 w = *reinterpret_cast<const uint2*>(p.packed + r * (p.k >> 1) + c * 8);
    float o[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t code = ((i < 8 ? w.x : w.y) >> (4 * (i & 7))) & 0xFu;
      const float t = kE2M1Table[code & 7u];
      const float val = __fmul_rn(t, (code & 8u) ? -1.0f : 1.0f);
      const float vs = __fmul_rn(val, scale);
      o[i] = p.div_mode == 0 ? __fmul_rn(vs, inv_gs) : __fdiv_rn(vs, p.gs);
    }
    float4* dst = reinterpret_cast<float4*>(p.out + r * p.k + c * 16);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
  }
}

__global__ void __launch_bounds__(256) nvfp4_swizzle_kernel(const uint8_t* in, int64_t rows, int64_t cols,
                                                            int64_t rows_pad, int64_t cols_pad, uint8_t* out) {
  const int64_t total = rows_pad * cols_pad;
  const int64_t c4 = cols_pad >> 2;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = b / cols_pad;
    const int64_t c = b - r * cols_pad;
    out[sf_swizzle_offset(r, c, c4)] = (r < rows && c < cols) ? in[r * cols + c] : 0;
  }
}

// max |x| as FP32 bits: for non-negative floats (and NaN, whose magnitude bits exceed +Inf) the
// unsigned order of the bit patterns is the numeric order, so atomicMax on the bits is a max.
// The same holds for the 16-bit patterns of |x| in f16 and bf16, so 16-bit inputs are reduced two
// elements per instruction (__vmaxu2 on the masked words) and widened to FP32 bits once at the end.
// Consecutive lanes read consecutive 16-byte vectors (512 contiguous bytes per warp and load), four
// loads in flight per thread.
template <int kInDtype>
__global__ void __launch_bounds__(256, 8) nvfp4_amax_kernel(const void* x, int64_t numel, unsigned int* out_bits) {
  constexpr int kPerVec = kInDtype == 2 ? 4 : 8;  // elements per 16-byte vector
  const uint4* xv = static_cast<const uint4*>(x);
  const int64_t nv = numel / kPerVec;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  uint32_t m = 0;  // f32: the max |x| bits; 16-bit: two running maxima, one per half-word
  auto fold = [&](const uint4& w) {
    if constexpr (kInDtype == 2) {
      m = max(m, max(max(w.x & 0x7FFFFFFFu, w.y & 0x7FFFFFFFu), max(w.z & 0x7FFFFFFFu, w.w & 0x7FFFFFFFu)));
    } else {
      m = __vmaxu2(m, __vmaxu2(__vmaxu2(w.x & 0x7FFF7FFFu, w.y & 0x7FFF7FFFu),
                               __vmaxu2(w.z & 0x7FFF7FFFu, w.w & 0x7FFF7FFFu)));
    }
  };
  int64_t v = gt;
  for (; v + 3 * stride < nv; v += 4 * stride) {
    const uint4 w0 = __ldg(xv + v), w1 = __ldg(xv + v + stride);
    const uint4 w2 = __ldg(xv + v + 2 * stride), w3 = __ldg(xv + v + 3 * stride);
    fold(w0);
    fold(w1);
    fold(w2);
    fold(w3);
  }
  for (; v < nv; v += stride) fold(__ldg(xv + v));
  if constexpr (kInDtype != 2) {
    const uint32_t h = max(m & 0xFFFFu, m >> 16);
    m = kInDtype == 1 ? h << 16 : __float_as_uint(__half2float(__ushort_as_half(static_cast<unsigned short>(h))));
  }
  // Tail (numel not a multiple of the vector), handled by the first threads.
  const int64_t tail0 = nv * kPerVec;
  if (gt < numel - tail0) {
    const int64_t e = tail0 + gt;
    float f;
    if constexpr (kInDtype == 2)
      f = static_cast<const float*>(x)[e];
    else if constexpr (kInDtype == 1)
      f = __uint_as_float(static_cast<uint32_t>(static_cast<const uint16_t*>(x)[e]) << 16);
    else
      f = __half2float(__ushort_as_half(static_cast<const uint16_t*>(x)[e]));
    m = max(m, __float_as_uint(f) & 0x7FFFFFFFu);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m != 0) atomicMax(out_bits, m);
}

}  // namespace g3
