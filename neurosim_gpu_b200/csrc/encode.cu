// encode.cu -- the fp8 (E4M3) and NVFP4 weight encoders on the device.
//
// Bit-exact to the reference quantizer (src/neurosim_gpu/precision.py:45-90):
//   fp8:   scale = max(amax / 448, FLT_MIN);
//          code  = e4m3_rn(clamp(w / scale, -448, 448))
//   nvfp4: g     = max(amax / 2688, FLT_MIN)                 (2688 = 6 * 448)
//          per 16 consecutive weights (zero-padded): bs = e4m3_rn(min(bamax / (6 g), 448))
//          code  = number of E2M1 midpoints {.25,.75,1.25,1.75,2.5,3.5,5} below
//                  |w| / (g * bs) (a tie counts for the odd-indexed midpoints,
//                  which lands it on the even code), sign bit 3 = signbit(w);
//          two codes per byte, the even-indexed weight in the low nibble.
// Every division is an IEEE division (div.rn), every product rounded once, as
// PyTorch computes them; e4m3_rn is the hardware round-to-nearest-even
// conversion with saturation (cvt.rn.satfinite.e4m3x2.f32).
//
// Launch 1 (amax_kernel): grid-stride max of |w| into a device word
//   (atomicMax on the bits: non-negative floats order like their bits).
// Launch 2 (fp8_kernel: 4 weights per thread, one 16-byte load, one 4-byte
//   store; nvfp4_kernel: one 16-weight block per thread, four 16-byte loads,
//   the block scale byte and 8 code bytes).  HBM-bound: 8 bytes read per weight
//   plus the codes written.
#include <algorithm>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kEncodeThreads = 256;
constexpr float kFloatMin = 1.17549435082228750797e-38f;  // FLT_MIN

__device__ __forceinline__ uint32_t e4m3_rn(float x) {
  unsigned short pair;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(pair) : "f"(0.0f), "f"(x));
  return pair & 0xffu;  // the second source lands in the low byte
}

// Exact value of an E4M3FN byte (finite codes; the encoders make no NaN).
__device__ __forceinline__ float e4m3_float(uint32_t code) { return e4m3_value(code); }

__global__ void __launch_bounds__(kEncodeThreads)
amax_kernel(const float* __restrict__ w, int64_t n, unsigned int* amax_bits) {
  unsigned int best = 0;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t quads = n >> 2;
  const bool vec = (reinterpret_cast<uintptr_t>(w) & 15) == 0;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    for (int64_t q = i; q < quads; q += stride) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(w) + q);
      best = max(best, __float_as_uint(fabsf(v.x)));
      best = max(best, __float_as_uint(fabsf(v.y)));
      best = max(best, __float_as_uint(fabsf(v.z)));
      best = max(best, __float_as_uint(fabsf(v.w)));
    }
    for (int64_t e = quads * 4 + i; e < n; e += stride) best = max(best, __float_as_uint(fabsf(__ldg(w + e))));
  } else {
    for (int64_t e = i; e < n; e += stride) best = max(best, __float_as_uint(fabsf(__ldg(w + e))));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, off));
  if ((threadIdx.x & 31) == 0 && best) atomicMax(amax_bits, best);
}

__global__ void __launch_bounds__(kEncodeThreads)
fp8_kernel(const float* __restrict__ w, int64_t n, const unsigned int* amax_bits,
           uint8_t* __restrict__ codes, float* global_scale) {
  const float amax = __uint_as_float(*amax_bits);
  const float scale = fmaxf(__fdiv_rn(amax, 448.0f), kFloatMin);
  if (blockIdx.x == 0 && threadIdx.x == 0) *global_scale = scale;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t quads = n >> 2;
  const bool vec = (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(codes) & 3) == 0;
  auto code_of = [scale](float v) {
    return e4m3_rn(fminf(448.0f, fmaxf(-448.0f, __fdiv_rn(v, scale))));
  };
  const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (vec) {
    for (int64_t q = first; q < quads; q += stride) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(w) + q);
      reinterpret_cast<uint32_t*>(codes)[q] =
          code_of(v.x) | (code_of(v.y) << 8) | (code_of(v.z) << 16) | (code_of(v.w) << 24);
    }
    for (int64_t e = quads * 4 + first; e < n; e += stride) codes[e] = static_cast<uint8_t>(code_of(__ldg(w + e)));
  } else {
    for (int64_t e = first; e < n; e += stride) codes[e] = static_cast<uint8_t>(code_of(__ldg(w + e)));
  }
}

// E2M1 code of a normalized magnitude (midpoint count, ties to the even code).
__device__ __forceinline__ uint32_t e2m1_code(float x) {
  return static_cast<uint32_t>(x > 0.25f) + static_cast<uint32_t>(x >= 0.75f) +
         static_cast<uint32_t>(x > 1.25f) + static_cast<uint32_t>(x >= 1.75f) +
         static_cast<uint32_t>(x > 2.5f) + static_cast<uint32_t>(x >= 3.5f) +
         static_cast<uint32_t>(x > 5.0f);
}

__global__ void __launch_bounds__(kEncodeThreads)
nvfp4_kernel(const float* __restrict__ w, int64_t n, const unsigned int* amax_bits,
             uint8_t* __restrict__ codes, uint8_t* __restrict__ block_scales,
             float* global_scale) {
  const float amax = __uint_as_float(*amax_bits);
  const float g = fmaxf(__fdiv_rn(amax, 2688.0f), kFloatMin);
  const float six_g = __fmul_rn(6.0f, g);
  if (blockIdx.x == 0 && threadIdx.x == 0) *global_scale = g;
  const int64_t blocks = (n + 15) >> 4;
  const int64_t packed = (n + 1) >> 1;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const bool vec = (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(codes) & 7) == 0;
  for (int64_t blk = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; blk < blocks;
       blk += stride) {
    const int64_t e0 = blk << 4;
    float v[16];
    if (vec && e0 + 16 <= n) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 x = __ldg(reinterpret_cast<const float4*>(w + e0) + q);
        v[4 * q] = x.x;
        v[4 * q + 1] = x.y;
        v[4 * q + 2] = x.z;
        v[4 * q + 3] = x.w;
      }
    } else {
#pragma unroll
      for (int k = 0; k < 16; ++k) v[k] = e0 + k < n ? __ldg(w + e0 + k) : 0.0f;  // zero padding
    }
    float bamax = 0.0f;
#pragma unroll
    for (int k = 0; k < 16; ++k) bamax = fmaxf(bamax, fabsf(v[k]));
    const uint32_t bs = e4m3_rn(fminf(__fdiv_rn(bamax, six_g), 448.0f));
    block_scales[blk] = static_cast<uint8_t>(bs);
    const float denominator = __fmul_rn(g, e4m3_float(bs));
    const float divisor = denominator > 0.0f ? denominator : 1.0f;
    unsigned long long word = 0ull;  // code k in bits [4k, 4k + 4)
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const unsigned long long code = e2m1_code(__fdiv_rn(fabsf(v[k]), divisor)) |
                                      ((__float_as_uint(v[k]) >> 31) << 3);
      word |= code << (4 * k);
    }
    uint8_t* out = codes + (blk << 3);
    if (vec && (blk << 3) + 8 <= packed) {
      *reinterpret_cast<unsigned long long*>(out) = word;
    } else {
      for (int k = 0; k < 8 && (blk << 3) + k < packed; ++k)
        out[k] = static_cast<uint8_t>(word >> (8 * k));
    }
  }
}

int grid_for(int64_t work, int sm_count) {
  const int64_t blocks = (work + kEncodeThreads - 1) / kEncodeThreads;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks, int64_t{sm_count} * 8)));
}

}  // namespace

cudaError_t launch_encode(int format, const float* weight, int64_t n, uint8_t* codes,
                          uint8_t* block_scales, float* global_scale, void* workspace,
                          cudaStream_t stream) {
  DeviceInfo info;
  cudaError_t err = device_info(&info);
  if (err != cudaSuccess) return err;
  auto* amax_bits = static_cast<unsigned int*>(workspace);
  err = cudaMemsetAsync(amax_bits, 0, sizeof(unsigned int), stream);
  if (err != cudaSuccess) return err;
  if (n > 0) {
    amax_kernel<<<grid_for((n + 3) / 4, info.sm_count), kEncodeThreads, 0, stream>>>(weight, n,
                                                                                  amax_bits);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
  }
  if (format == NSB_WEIGHT_E4M3) {
    fp8_kernel<<<grid_for((n + 3) / 4, info.sm_count), kEncodeThreads, 0, stream>>>(
        weight, n, amax_bits, codes, global_scale);
  } else {
    nvfp4_kernel<<<grid_for((n + 15) / 16, info.sm_count), kEncodeThreads, 0, stream>>>(
        weight, n, amax_bits, codes, block_scales, global_scale);
  }
  return cudaGetLastError();
}

}  // namespace nsb
