// NVFP4 quantiser, dequantiser, scale swizzle and tensor amax for sm_100a.
//
// The quantiser reproduces nvfp4_gemm_cute/quant.py:41-59 bit for bit:
//   xb    = float(x) * gs                                   (one FP32 multiply)
//   amax  = max |xb| over 16 consecutive K elements         (NaN propagates, like torch.amax)
//   scale = e4m3fn(amax / 6)  round-to-nearest-even, overflow -> NaN (no saturation)
//   q     = scale > 0 ? xb / scale : 0                      (IEEE division)
//   code  = argmin_i (|min(|q|, 6) - E2M1[i]| + (i odd) * 1e-6f), first index on ties
//           | 8 if q < 0                                     (quant.py:15-28)
// The argmin runs on the two table entries that bracket |q|: the distance to every other entry
// is larger by at least 0.5, far more than the 1e-6 penalty, and FP32 subtraction is monotone,
// so the bracketing pair always holds the minimum. Both distances are computed with the same
// FP32 operations as the reference (no contraction), so ties resolve identically.
//
// One thread owns one 16-element scale block. Consecutive threads own consecutive blocks of
// the row-major input, so loads (32 or 64 bytes per thread), code stores (8 bytes) and linear
// scale stores are coalesced; the swizzled scale byte goes to its 128x4-tile position.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

namespace g3 {

// FP32 -> E4M3 (fn variant: bias 7, max 448, 0x7F/0xFF = NaN, no infinities), round to nearest
// even, non-saturating: anything that rounds above 448 becomes NaN.
__device__ __forceinline__ uint32_t f32_to_e4m3_rn(float f) {
  const uint32_t u = __float_as_uint(f);
  const uint32_t sign = (u >> 24) & 0x80u;
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x43E80000u) return sign | 0x7Fu;  // NaN, Inf, or |f| > 464 (rounds past 448)
  if (a >= 0x3C800000u) {                    // |f| >= 2^-6: normal E4M3
    const uint32_t r = (a + 0x7FFFFu + ((a >> 20) & 1u)) >> 20;  // keep 3 mantissa bits, RNE
    return sign | (r - (120u << 3));                             // rebias exponent 127 -> 7
  }
  // Subnormal E4M3: multiples of 2^-9. f * 512 is exact; rintf rounds half to even.
  const uint32_t q = static_cast<uint32_t>(rintf(__uint_as_float(a) * 512.0f));
  return sign | q;  // q == 8 is the smallest normal (0x08), which is also correct
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t b) {
  const uint32_t sign = (b & 0x80u) << 24;
  const uint32_t e = (b >> 3) & 0xFu;
  const uint32_t m = b & 7u;
  if (e == 0xFu && m == 7u) return __uint_as_float(sign | 0x7FC00000u);
  if (e == 0) return __uint_as_float(sign | __float_as_uint(static_cast<float>(m) * 0.001953125f));
  return __uint_as_float(sign | ((e + 120u) << 23) | (m << 20));
}

__device__ __constant__ float kE2M1Table[9] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f, 6.0f};

// Nearest E2M1 magnitude code (0-7) of q, with the reference's tie rule.
__device__ __forceinline__ uint32_t e2m1_code(float q) {
  const float mag = fminf(fabsf(q), 6.0f);  // torch clamp(max=6); NaN handled by the caller
  const uint32_t i = (mag >= 0.5f) + (mag >= 1.0f) + (mag >= 1.5f) + (mag >= 2.0f) + (mag >= 3.0f) +
                     (mag >= 4.0f) + (mag >= 6.0f);
  if (i == 7u) return 7u;
  const float pen = 9.99999997e-07f;  // float32(1e-6), added to odd codes
  const float d_lo = __fadd_rn(__fsub_rn(mag, kE2M1Table[i]), (i & 1u) ? pen : 0.0f);
  const float d_hi = __fadd_rn(__fsub_rn(kE2M1Table[i + 1], mag), ((i + 1u) & 1u) ? pen : 0.0f);
  return d_hi < d_lo ? i + 1u : i;
}

// Byte offset of scale (row, col) in the 128x4 swizzled layout with `c4` 4-column groups.
__device__ __forceinline__ int64_t sf_swizzle_offset(int64_t row, int64_t col, int64_t c4) {
  return ((row >> 7) * c4 + (col >> 2)) * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (col & 3);
}

template <int kInDtype>  // 0 = f16, 1 = bf16, 2 = f32
__device__ __forceinline__ void load16(const void* base, int64_t elem, float (&v)[16]) {
  if constexpr (kInDtype == 2) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(base) + elem);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 f = __ldg(p + i);
      v[4 * i] = f.x;
      v[4 * i + 1] = f.y;
      v[4 * i + 2] = f.z;
      v[4 * i + 3] = f.w;
    }
  } else {
    const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(base) + elem);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const uint4 w = __ldg(p + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (kInDtype == 1) {
          v[8 * i + 2 * j] = __uint_as_float(ws[j] << 16);
          v[8 * i + 2 * j + 1] = __uint_as_float(ws[j] & 0xFFFF0000u);
        } else {
          v[8 * i + 2 * j] = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[j] & 0xFFFFu)));
          v[8 * i + 2 * j + 1] = __half2float(__ushort_as_half(static_cast<unsigned short>(ws[j] >> 16)));
        }
      }
    }
  }
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

template <int kInDtype>
__global__ void __launch_bounds__(256) nvfp4_quantize_kernel(const QuantParams p) {
  const float gs = resolve_global_scale(p);
  if (p.gs_out != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *p.gs_out = gs;
  const float inv6 = 0.166666672f;  // fl(1/6): what torch on CUDA multiplies by for "/ 6.0"
  const int64_t total = p.rows_pad * p.cols_pad;
  const int64_t c4 = p.cols_pad >> 2;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = b / p.cols_pad;
    const int64_t c = b - r * p.cols_pad;
    uint32_t sf = 0;
    if (r < p.rows && c < p.cols) {
      float v[16];
      load16<kInDtype>(p.x, r * p.k + c * 16, v);
      float amax = 0.0f;
      bool nan = false;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        v[i] = __fmul_rn(v[i], gs);
        const float a = fabsf(v[i]);
        nan |= (a != a);
        amax = fmaxf(amax, a);
      }
      const float s = p.div_mode == 0 ? __fmul_rn(amax, inv6) : __fdiv_rn(amax, 6.0f);
      sf = nan ? 0x7Fu : f32_to_e4m3_rn(s);
      const float denom = e4m3_to_f32(sf);
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float q = denom > 0.0f ? __fdiv_rn(v[i], denom) : 0.0f;
        const uint32_t code = e2m1_code(q) | (q < 0.0f ? 8u : 0u);
        if (i < 8)
          lo |= code << (4 * i);
        else
          hi |= code << (4 * (i - 8));
      }
      *reinterpret_cast<uint2*>(p.packed + r * (p.k >> 1) + c * 8) = make_uint2(lo, hi);
      if (p.sf_lin != nullptr) p.sf_lin[r * p.cols + c] = static_cast<uint8_t>(sf);
    }
    p.sf_swz[sf_swizzle_offset(r, c, c4)] = static_cast<uint8_t>(sf);
  }
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
template <int kInDtype>
__global__ void __launch_bounds__(256) nvfp4_amax_kernel(const void* x, int64_t numel, unsigned int* out_bits) {
  uint32_t m = 0;
  const int64_t nvec = numel / 16;
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < nvec;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[16];
    load16<kInDtype>(x, b * 16, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = max(m, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  }
  // Tail (numel not a multiple of 16), handled by the first threads.
  const int64_t tail0 = nvec * 16;
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
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
