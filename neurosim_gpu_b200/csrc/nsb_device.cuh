// nsb_device.cuh -- device-side building blocks shared by the tick kernels.
//
// Contents: strided [B,N] operand access, the three-state pointwise update,
// streaming (read-once) vector loads, and in-register decoders for the four
// CSR weight formats.  Target: sm_100a only.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "neurosim_b200.h"

namespace nsb {

// ---------------------------------------------------------------------------
// Operands
// ---------------------------------------------------------------------------

// A [B,N] float32 operand; data == nullptr means "constant scalar".
struct View {
  const float* data;
  int64_t sb, sn;
  float scalar;
  __device__ __forceinline__ float at(int64_t b, int64_t n) const {
    return data ? __ldg(data + b * sb + n * sn) : scalar;
  }
};

struct Out {
  float* data;
  int64_t sb, sn;
  __device__ __forceinline__ void put(int64_t b, int64_t n, float v) const {
    data[b * sb + n * sn] = v;
  }
};

struct Params {
  const float* data[6];
  int64_t stride[6];
  __device__ __forceinline__ float at(int i, int64_t n) const {
    return __ldg(data[i] + n * stride[i]);
  }
};

struct TickArgs {
  int64_t batch, neurons;
  View s, d, a, u, v;
  Params p;
};

struct TickOut {
  Out s, d, a;
};

// ---------------------------------------------------------------------------
// The pointwise update.  Every product and sum is rounded on its own (no FMA
// contraction), in the order of the reference's PyTorch ops
// (compartmental.py:168-183, dynamics.py:52-61):
//   d' = rd*d + (1-rd)*tanh(j + v)
//   x  = ((1-c)*j + c*d') - k*a
//   s' = clamp(alpha*s + (1-alpha)*(gain*tanh(x + u)), 0, 1)
//   a' = ra*a + (1-ra)*s'
// ---------------------------------------------------------------------------
struct Update {
  float s, d, a;
};

__device__ __forceinline__ Update advance(float j, float s, float d, float a, float u,
                                          float v, float alpha, float gain, float rd,
                                          float ra, float c, float k) {
  Update r;
  r.d = __fadd_rn(__fmul_rn(rd, d), __fmul_rn(__fsub_rn(1.0f, rd), tanhf(__fadd_rn(j, v))));
  const float x = __fsub_rn(__fadd_rn(__fmul_rn(__fsub_rn(1.0f, c), j), __fmul_rn(c, r.d)),
                            __fmul_rn(k, a));
  const float eq = __fmul_rn(gain, tanhf(__fadd_rn(x, u)));
  const float next = __fadd_rn(__fmul_rn(alpha, s), __fmul_rn(__fsub_rn(1.0f, alpha), eq));
  r.s = fminf(1.0f, fmaxf(0.0f, next));
  r.a = __fadd_rn(__fmul_rn(ra, a), __fmul_rn(__fsub_rn(1.0f, ra), r.s));
  return r;
}

__device__ __forceinline__ Update advance_at(const TickArgs& t, float j, int64_t b, int64_t n) {
  return advance(j, t.s.at(b, n), t.d.at(b, n), t.a.at(b, n), t.u.at(b, n), t.v.at(b, n),
                 t.p.at(0, n), t.p.at(1, n), t.p.at(2, n), t.p.at(3, n), t.p.at(4, n),
                 t.p.at(5, n));
}

// ---------------------------------------------------------------------------
// Streaming loads: each edge byte is read exactly once per tick, so the edge
// arrays bypass L1 and are marked evict-first in L2.  That keeps L1/L2 for
// the gathered source state, which every edge re-reads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

__device__ __forceinline__ int4 stream_load_v4(const int4* p, uint64_t pol) {
  int4 r;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v4.s32 {%0,%1,%2,%3}, [%4], %5;"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint2 stream_load_v2(const uint2* p, uint64_t pol) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t stream_load_u32(const uint32_t* p, uint64_t pol) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t stream_load_u16(const uint16_t* p, uint64_t pol) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;"
               : "=h"(r)
               : "l"(p), "l"(pol));
  return r;
}

// ---------------------------------------------------------------------------
// Number formats, decoded from their definitions.
// ---------------------------------------------------------------------------

// OCP FP8 E4M3FN: 1 sign, 4 exponent bits (bias 7), 3 mantissa bits, no
// infinities, S.1111.111 = NaN.  Exact conversion to float32.
__device__ __forceinline__ float e4m3_value(uint32_t code) {
  const uint32_t em = code & 0x7fu;
  const uint32_t sign = (code & 0x80u) << 24;
  // Normal: move the 7 exponent+mantissa bits under the float32 fields and
  // rebias the exponent (7 -> 127).  Subnormal: mantissa * 2^-9 (exact).
  const float normal = __uint_as_float((em + (120u << 3)) << 20);
  const float subnormal = static_cast<float>(em) * 0.001953125f;
  float mag = em >= 8u ? normal : subnormal;
  mag = em == 0x7fu ? __uint_as_float(0x7fc00000u) : mag;
  return __uint_as_float(__float_as_uint(mag) | sign);
}

// E2M1 (FP4): 1 sign, 2 exponent bits (bias 1), 1 mantissa bit:
// magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6.  Returns the signed value.
__device__ __forceinline__ float e2m1_value(uint32_t code) {
  const uint32_t c = code & 7u;
  const float normal = __uint_as_float((((c >> 1) + 126u) << 23) | ((c & 1u) << 22));
  const float mag = c >= 2u ? normal : 0.5f * static_cast<float>(c);
  return __uint_as_float(__float_as_uint(mag) | ((code & 8u) << 28));
}

// ---------------------------------------------------------------------------
// Weight readers.  `quad(c, w)` fills the weights of edges 4c..4c+3 from one
// aligned vector load (the caller guarantees 4c+4 <= M and aligned base
// pointers); `one(e)` reads a single edge (tails and unaligned bases).
//
// The decoded value equals the reference quantizer's dequantized weight bit
// for bit: fp8 -> e4m3(code) * g ; nvfp4 -> e2m1(code) * (e4m3(block) * g)
// (precision.py:102-109).
// ---------------------------------------------------------------------------
struct WeightsF32 {
  const float* w;
  __device__ __forceinline__ void quad(int64_t c, float (&out)[4], uint64_t pol) const {
    const int4 r = stream_load_v4(reinterpret_cast<const int4*>(w) + c, pol);
    out[0] = __int_as_float(r.x);
    out[1] = __int_as_float(r.y);
    out[2] = __int_as_float(r.z);
    out[3] = __int_as_float(r.w);
  }
  __device__ __forceinline__ float one(int64_t e) const { return __ldg(w + e); }
};

struct WeightsF16 {
  const __half* w;
  __device__ __forceinline__ void quad(int64_t c, float (&out)[4], uint64_t pol) const {
    const uint2 r = stream_load_v2(reinterpret_cast<const uint2*>(w) + c, pol);
    out[0] = __half2float(__ushort_as_half(static_cast<unsigned short>(r.x & 0xffffu)));
    out[1] = __half2float(__ushort_as_half(static_cast<unsigned short>(r.x >> 16)));
    out[2] = __half2float(__ushort_as_half(static_cast<unsigned short>(r.y & 0xffffu)));
    out[3] = __half2float(__ushort_as_half(static_cast<unsigned short>(r.y >> 16)));
  }
  __device__ __forceinline__ float one(int64_t e) const { return __half2float(w[e]); }
};

struct WeightsE4M3 {
  const uint8_t* codes;
  const float* global;
  __device__ __forceinline__ void quad(int64_t c, float (&out)[4], uint64_t pol) const {
    const uint32_t r = stream_load_u32(reinterpret_cast<const uint32_t*>(codes) + c, pol);
    const float g = __ldg(global);
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = __fmul_rn(e4m3_value((r >> (8 * k)) & 0xffu), g);
  }
  __device__ __forceinline__ float one(int64_t e) const {
    return __fmul_rn(e4m3_value(codes[e]), __ldg(global));
  }
};

struct WeightsNVFP4 {
  const uint8_t* codes;   // two E2M1 codes per byte, even edge in the low nibble
  const uint8_t* scales;  // one E4M3 scale per 16 edges
  const float* global;
  __device__ __forceinline__ void quad(int64_t c, float (&out)[4], uint64_t pol) const {
    const uint32_t r = stream_load_u16(reinterpret_cast<const uint16_t*>(codes) + c, pol);
    // Edges 4c..4c+3 share block (4c)/16 = c/4.
    const float block = __fmul_rn(e4m3_value(__ldg(scales + (c >> 2))), __ldg(global));
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = __fmul_rn(e2m1_value((r >> (4 * k)) & 15u), block);
  }
  __device__ __forceinline__ float one(int64_t e) const {
    const uint32_t code = (codes[e >> 1] >> ((e & 1) * 4)) & 15u;
    const float block = __fmul_rn(e4m3_value(__ldg(scales + (e >> 4))), __ldg(global));
    return __fmul_rn(e2m1_value(code), block);
  }
};

}  // namespace nsb
