// tick.cu -- the fused matrix tick: CSR SpMV j = W @ s plus the three-state update.
//
// Work decomposition
//   * A group of G lanes (G = 4, 8, 16 or 32) owns one destination row n and
//     every batch row of the current batch tile (BT <= 8 batch rows).  The
//     row's edges are therefore streamed from HBM once per batch tile, not once
//     per batch row as in the reference kernel (csrc/compartmental.cu:121-140).
//   * Edges are read as 4-edge chunks aligned to the array start: the chunk of
//     edges 4c..4c+3 is one 16-byte col load plus one vector weight load
//     (16 B fp32, 8 B fp16, 4 B e4m3, 2 B nvfp4).  Lanes of a group take
//     consecutive chunks, so a group issues contiguous, coalesced loads;
//     edges of the chunk outside [rowptr[n], rowptr[n+1]) are masked.
//   * The gathered source state x[b, col] goes through L1/L2 (it is re-read by
//     every edge), while the edge stream bypasses L1 and is evict-first in L2.
//   * Partial sums are reduced with xor shuffles inside the group; lane
//     (b mod G) of the group then applies the pointwise update for batch row b
//     and writes s', d', a' (or the bare product for nsb_csr_propagate).
//   * The grid is persistent over rows: SMs x resident blocks, grid-stride.
//
// Batched variant (csr_batch_kernel, every B >= 2; fastest when the batch rows
// of a source are contiguous, the [N, B] state layout the runtime keeps):
//   * G lanes (8, 16 or 32, from the mean degree) own one destination row and a
//     tile of BT <= 8 batch rows.  Lane l of the group takes the row's edges
//     e0 + l, e0 + l + G, ... (two in flight), and for each one loads the
//     BT batch values of its source: with the [N, B] layout that is ONE vector
//     load of BT contiguous floats (for BT = 8 a 256-bit load, one 32-byte
//     sector), otherwise BT scalar loads -- the arithmetic is the same either
//     way, so the result does not depend on the state's layout.
//   * Each lane accumulates BT sums in CSR order over its edges.  The group
//     then reduces its BT x G partial sums with a transposing butterfly (step
//     s halves the values a lane keeps, exchanging the other half with the
//     lane G >> (s + 1) away), ending with batch row b on lanes
//     b * G / BT .. (b + 1) * G / BT - 1; a fixed xor tree finishes the sum.
//   * The first lane of each batch row's lanes applies the pointwise update;
//     with the [N, B] layout the BT updating lanes write one contiguous span.
#include <algorithm>
#include <type_traits>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kThreads = 256;

bool aligned(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
}

template <int G, int BT, bool UPDATE, typename W>
__global__ void __launch_bounds__(kThreads)
csr_tick_kernel(TickArgs t, View x, const int32_t* __restrict__ rowptr,
                const int32_t* __restrict__ col, int64_t n_edges, W weights, bool vec,
                TickOut out, Out product) {
  static_assert(32 % G == 0, "group width must divide the warp");
  constexpr int kRowsPerWarp = 32 / G;
  const int lane = threadIdx.x & 31;
  const int lg = lane % G;
  const int64_t neurons = t.neurons;
  const int64_t batch = t.batch;
  const int64_t b0 = static_cast<int64_t>(blockIdx.y) * BT;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const uint64_t pol = evict_first_policy();
  const float* __restrict__ xs = x.data;

  for (int64_t base = warp * kRowsPerWarp; base < neurons; base += n_warps * kRowsPerWarp) {
    const int64_t n = base + lane / G;
    // -0.0 is the exact additive identity: a one-term row keeps a signed zero.
    float acc[BT];
#pragma unroll
    for (int b = 0; b < BT; ++b) acc[b] = -0.0f;

    if (n < neurons) {
      const int64_t e0 = rowptr[n];
      const int64_t e1 = rowptr[n + 1];
      if (vec) {
        const int64_t c_end = (e1 + 3) >> 2;
        for (int64_t c = (e0 >> 2) + lg; c < c_end; c += G) {
          const int64_t e = c << 2;
          int cols[4];
          float w[4];
          if (e + 4 <= n_edges) {
            const int4 cc = stream_load_v4(reinterpret_cast<const int4*>(col) + c, pol);
            cols[0] = cc.x;
            cols[1] = cc.y;
            cols[2] = cc.z;
            cols[3] = cc.w;
            weights.quad(c, w, pol);
          } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const bool in = e + k < n_edges;
              cols[k] = in ? __ldg(col + e + k) : 0;
              w[k] = in ? weights.one(e + k) : 0.0f;
            }
          }
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            if (e + k >= e0 && e + k < e1) {
              const float* xc = xs + static_cast<int64_t>(cols[k]) * x.sn;
#pragma unroll
              for (int b = 0; b < BT; ++b)
                if (b0 + b < batch) acc[b] = fmaf(w[k], __ldg(xc + (b0 + b) * x.sb), acc[b]);
            }
          }
        }
      } else {
        for (int64_t e = e0 + lg; e < e1; e += G) {
          const float w = weights.one(e);
          const float* xc = xs + static_cast<int64_t>(__ldg(col + e)) * x.sn;
#pragma unroll
          for (int b = 0; b < BT; ++b)
            if (b0 + b < batch) acc[b] = fmaf(w, __ldg(xc + (b0 + b) * x.sb), acc[b]);
        }
      }
    }

#pragma unroll
    for (int off = G / 2; off > 0; off >>= 1) {
#pragma unroll
      for (int b = 0; b < BT; ++b) acc[b] += __shfl_xor_sync(0xffffffffu, acc[b], off);
    }

    if (n < neurons) {
#pragma unroll
      for (int b = 0; b < BT; ++b) {
        if (b % G == lg && b0 + b < batch) {
          if constexpr (UPDATE) {
            const Update r = advance_at(t, acc[b], b0 + b, n);
            out.s.put(b0 + b, n, r.s);
            out.d.put(b0 + b, n, r.d);
            out.a.put(b0 + b, n, r.a);
          } else {
            product.put(b0 + b, n, acc[b]);
          }
        }
      }
    }
  }
}

// BT floats of one source for the batch tile: one vector load from a
// BT * 4-byte aligned address (VEC), else BT strided scalar loads (entries
// past the batch read as 0).  The 32-byte gathers of B = 8 do not allocate
// in L1: a warp's 32 random sources rarely share a line, and the tag lookups
// of allocating loads bound the kernel (166k / 25M, B = 8: 128.1 -> 125.3 us
// per tick).
template <int BT, bool VEC>
__device__ __forceinline__ void load_batch(const float* p, int64_t sb, int valid, float (&v)[BT]) {
  if constexpr (VEC && BT == 8) {
    asm("ld.global.nc.L1::no_allocate.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]),
          "=f"(v[7])
        : "l"(p));
  } else if constexpr (VEC && BT == 4) {
    asm("ld.global.nc.v4.f32 {%0,%1,%2,%3}, [%4];"
        : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3])
        : "l"(p));
  } else if constexpr (VEC && BT == 2) {
    asm("ld.global.nc.v2.f32 {%0,%1}, [%2];" : "=f"(v[0]), "=f"(v[1]) : "l"(p));
  } else {
#pragma unroll
    for (int b = 0; b < BT; ++b) v[b] = b < valid ? __ldg(p + b * sb) : 0.0f;
  }
}

// One edge's weight: the edge stream is read once per tick, so fp32 weights
// bypass L1 and are evict-first in L2 (the narrower formats go through
// their decoders).
template <typename W>
__device__ __forceinline__ float edge_weight(const W& w, int64_t e, uint64_t pol) {
  if constexpr (std::is_same<W, WeightsF32>::value) {
    float r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.f32 %0, [%1], %2;"
                 : "=f"(r)
                 : "l"(w.w + e), "l"(pol));
    return r;
  } else {
    return w.one(e);
  }
}

template <int BT, int G, bool UPDATE, bool VEC, typename W>
__global__ void __launch_bounds__(kThreads)
csr_batch_kernel(TickArgs t, View x, const int32_t* __restrict__ rowptr,
                 const int32_t* __restrict__ col, W weights, TickOut out, Out product) {
  static_assert(G >= BT && G <= 32 && 32 % G == 0, "group width");
  constexpr int kPerBatch = G / BT;  // lanes of a group that end with one batch row
  const int lane = threadIdx.x & 31;
  const int lg = lane % G;
  const int64_t neurons = t.neurons;
  const int64_t b0 = static_cast<int64_t>(blockIdx.y) * BT;
  const int valid = static_cast<int>(t.batch - b0 < BT ? t.batch - b0 : BT);
  const int64_t group = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / G;
  const int64_t n_groups = static_cast<int64_t>(gridDim.x) * blockDim.x / G;
  const uint64_t pol = evict_first_policy();
  const float* __restrict__ xb = x.data + b0 * x.sb;

  for (int64_t base = group - lane / G; base < neurons; base += n_groups) {
    const int64_t n = base + lane / G;  // the groups of a warp take consecutive rows
    float acc[BT];
#pragma unroll
    for (int b = 0; b < BT; ++b) acc[b] = -0.0f;  // -0.0 is the exact additive identity
    if (n < neurons) {
      const int64_t e1 = __ldg(rowptr + n + 1);
      int64_t e = __ldg(rowptr + n) + lg;
      for (; e + G < e1; e += 2 * G) {  // two edges per lane in flight
        const int c0 = static_cast<int>(stream_load_u32(reinterpret_cast<const uint32_t*>(col + e), pol));
        const int c1 = static_cast<int>(stream_load_u32(reinterpret_cast<const uint32_t*>(col + e + G), pol));
        const float w0 = edge_weight(weights, e, pol);
        const float w1 = edge_weight(weights, e + G, pol);
        float v0[BT], v1[BT];
        load_batch<BT, VEC>(xb + static_cast<int64_t>(c0) * x.sn, x.sb, valid, v0);
        load_batch<BT, VEC>(xb + static_cast<int64_t>(c1) * x.sn, x.sb, valid, v1);
#pragma unroll
        for (int b = 0; b < BT; ++b) acc[b] = fmaf(w0, v0[b], acc[b]);
#pragma unroll
        for (int b = 0; b < BT; ++b) acc[b] = fmaf(w1, v1[b], acc[b]);
      }
      if (e < e1) {
        const int c0 = static_cast<int>(stream_load_u32(reinterpret_cast<const uint32_t*>(col + e), pol));
        const float w0 = edge_weight(weights, e, pol);
        float v0[BT];
        load_batch<BT, VEC>(xb + static_cast<int64_t>(c0) * x.sn, x.sb, valid, v0);
#pragma unroll
        for (int b = 0; b < BT; ++b) acc[b] = fmaf(w0, v0[b], acc[b]);
      }
    }
    // Transposing butterfly: after step s a lane keeps BT >> (s + 1) sums; the
    // upper lane of each pair keeps the upper half of the values.
#pragma unroll
    for (int s = 0; (BT >> s) > 1; ++s) {
      const int off = G >> (s + 1);
      const int half = (BT >> s) / 2;
      const bool upper = (lg & off) != 0;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = upper ? acc[i] : acc[half + i];
        const float keep = upper ? acc[half + i] : acc[i];
        acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
#pragma unroll
    for (int off = kPerBatch / 2; off > 0; off >>= 1)
      acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], off);
    const int b = lg / kPerBatch;
    if (n < neurons && lg % kPerBatch == 0 && b < valid) {
      if constexpr (UPDATE) {
        const Update r = advance_at(t, acc[0], b0 + b, n);
        out.s.put(b0 + b, n, r.s);
        out.d.put(b0 + b, n, r.d);
        out.a.put(b0 + b, n, r.a);
      } else {
        product.put(b0 + b, n, acc[0]);
      }
    }
  }
}

template <typename K>
int resident_blocks(K kernel) {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kThreads, 0) != cudaSuccess)
    blocks = 1;
  return std::max(blocks, 1);
}

template <int G, int BT, bool UPDATE, typename W>
cudaError_t launch_variant(const TickArgs& t, const View& x, const Csr& csr, const W& weights,
                           bool vec, const TickOut& out, const Out& product,
                           cudaStream_t stream) {
  auto kernel = csr_tick_kernel<G, BT, UPDATE, W>;
  static int occupancy[64] = {0};  // per device ordinal, filled on first use
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  DeviceInfo info;
  err = device_info(&info);
  if (err != cudaSuccess) return err;
  int& occ = occupancy[device & 63];
  if (occ == 0) occ = resident_blocks(kernel);
  const int64_t rows_per_block = (kThreads / 32) * (32 / G);
  const int64_t needed = (t.neurons + rows_per_block - 1) / rows_per_block;
  const int64_t cap = static_cast<int64_t>(info.sm_count) * occ;
  const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, std::min(needed, cap))),
                  static_cast<unsigned>((t.batch + BT - 1) / BT));
  kernel<<<grid, kThreads, 0, stream>>>(t, x, csr.rowptr, csr.col, csr.n_edges, weights, vec,
                                        out, product);
  return cudaGetLastError();
}

template <int BT, int G, bool UPDATE, bool VEC, typename W>
cudaError_t launch_batch_variant(const TickArgs& t, const View& x, const Csr& csr, const W& weights,
                                 const TickOut& out, const Out& product, cudaStream_t stream) {
  auto kernel = csr_batch_kernel<BT, G, UPDATE, VEC, W>;
  static int occupancy[64] = {0};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  DeviceInfo info;
  err = device_info(&info);
  if (err != cudaSuccess) return err;
  int& occ = occupancy[device & 63];
  if (occ == 0) occ = resident_blocks(kernel);
  const int64_t rows_per_block = kThreads / G;
  const int64_t needed = (t.neurons + rows_per_block - 1) / rows_per_block;
  const int64_t cap = static_cast<int64_t>(info.sm_count) * occ;
  const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, std::min(needed, cap))),
                  static_cast<unsigned>((t.batch + BT - 1) / BT));
  kernel<<<grid, kThreads, 0, stream>>>(t, x, csr.rowptr, csr.col, weights, out, product);
  return cudaGetLastError();
}

template <int BT, bool UPDATE, typename W>
cudaError_t dispatch_batch_tile(const TickArgs& t, const View& x, const Csr& csr, const W& w,
                                int width, const TickOut& out, const Out& product,
                                cudaStream_t stream) {
  // One vector load per (edge, batch tile) needs every tile full and its BT
  // floats contiguous and BT * 4-byte aligned.
  const bool vec = x.sb == 1 && x.sn % BT == 0 && t.batch % BT == 0 &&
                   aligned(x.data, static_cast<uintptr_t>(BT) * 4);
  // Lanes per row: the caller's width (8 / 16 / 32; smaller means 8), else
  // from the mean degree (each lane takes two edges per step).  The lanes fix
  // a row's summation order, so the row blocks of a sharded graph pass the
  // whole graph's choice.
  const double degree = static_cast<double>(csr.n_edges) / static_cast<double>(std::max<int64_t>(t.neurons, 1));
  const int lanes = width > 0 ? (width <= 8 ? 8 : width <= 16 ? 16 : 32)
                              : degree <= 24.0 ? 8 : degree <= 64.0 ? 16 : 32;
#define NSB_BATCH(G)                                                                          \
  return vec ? launch_batch_variant<BT, G, UPDATE, true>(t, x, csr, w, out, product, stream)  \
             : launch_batch_variant<BT, G, UPDATE, false>(t, x, csr, w, out, product, stream);
  if (lanes == 8) { NSB_BATCH(8) }
  if (lanes == 16) { NSB_BATCH(16) }
  NSB_BATCH(32)
#undef NSB_BATCH
}

template <bool UPDATE, typename W>
cudaError_t dispatch_batch(const TickArgs& t, const View& x, const Csr& csr, const W& w,
                           int width, const TickOut& out, const Out& product,
                           cudaStream_t stream) {
  if (t.batch <= 2)
    return dispatch_batch_tile<2, UPDATE>(t, x, csr, w, width, out, product, stream);
  if (t.batch <= 4)
    return dispatch_batch_tile<4, UPDATE>(t, x, csr, w, width, out, product, stream);
  return dispatch_batch_tile<8, UPDATE>(t, x, csr, w, width, out, product, stream);
}

template <bool UPDATE, typename W>
cudaError_t dispatch_group(const TickArgs& t, const View& x, const Csr& csr, const W& w,
                           bool vec, int width, const TickOut& out, const Out& product,
                           cudaStream_t stream) {
  const int64_t batch = t.batch;
  // B >= 2: the batch-cooperative kernel, whatever the source strides, so the
  // summation order (and the result) does not depend on the state's layout.
  // With the [N, B] layout (batch stride 1) its gathers are one sector per edge.
  if (batch >= 2 && x.data)
    return dispatch_batch<UPDATE>(t, x, csr, w, width, out, product, stream);
#define NSB_BT(G)                                                                      \
  if (batch <= 1) return launch_variant<G, 1, UPDATE>(t, x, csr, w, vec, out, product, stream); \
  if (batch <= 2) return launch_variant<G, 2, UPDATE>(t, x, csr, w, vec, out, product, stream); \
  if (batch <= 4) return launch_variant<G, 4, UPDATE>(t, x, csr, w, vec, out, product, stream); \
  return launch_variant<G, 8, UPDATE>(t, x, csr, w, vec, out, product, stream);
  if (width == 0) width = choose_group_width(csr.n_edges, t.neurons);
  switch (width) {
    case 4: { NSB_BT(4) }
    case 8: { NSB_BT(8) }
    case 16: { NSB_BT(16) }
    default: { NSB_BT(32) }
  }
#undef NSB_BT
}

}  // namespace

cudaError_t device_info(DeviceInfo* info) {
  static int sm_counts[64] = {0};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  int& sms = sm_counts[device & 63];
  if (sms == 0) {
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) return err;
  }
  info->sm_count = sms;
  return cudaSuccess;
}

int choose_group_width(int64_t n_edges, int64_t neurons) {
  // Chunks of 4 edges per lane, plus about one partial chunk at each row end.
  const double chunks = static_cast<double>(n_edges) / static_cast<double>(std::max<int64_t>(neurons, 1)) / 4.0 + 1.0;
  if (chunks > 16.0) return 32;
  if (chunks > 8.0) return 16;
  if (chunks > 3.0) return 8;
  return 4;
}

cudaError_t launch_csr(const TickArgs& t, const View& x, const Csr& csr, int width, bool update,
                       const TickOut& out, const Out& product, cudaStream_t stream) {
  const bool col_ok = aligned(csr.col, 16);
  switch (csr.format) {
    case NSB_WEIGHT_F16: {
      WeightsF16 w{static_cast<const __half*>(csr.weight)};
      const bool vec = col_ok && aligned(csr.weight, 8);
      return update ? dispatch_group<true>(t, x, csr, w, vec, width, out, product, stream)
                    : dispatch_group<false>(t, x, csr, w, vec, width, out, product, stream);
    }
    case NSB_WEIGHT_E4M3: {
      WeightsE4M3 w{static_cast<const uint8_t*>(csr.weight), csr.global_scale};
      const bool vec = col_ok && aligned(csr.weight, 4);
      return update ? dispatch_group<true>(t, x, csr, w, vec, width, out, product, stream)
                    : dispatch_group<false>(t, x, csr, w, vec, width, out, product, stream);
    }
    case NSB_WEIGHT_NVFP4: {
      WeightsNVFP4 w{static_cast<const uint8_t*>(csr.weight), csr.block_scales, csr.global_scale};
      const bool vec = col_ok && aligned(csr.weight, 2);
      return update ? dispatch_group<true>(t, x, csr, w, vec, width, out, product, stream)
                    : dispatch_group<false>(t, x, csr, w, vec, width, out, product, stream);
    }
    default: {
      WeightsF32 w{static_cast<const float*>(csr.weight)};
      const bool vec = col_ok && aligned(csr.weight, 16);
      return update ? dispatch_group<true>(t, x, csr, w, vec, width, out, product, stream)
                    : dispatch_group<false>(t, x, csr, w, vec, width, out, product, stream);
    }
  }
}

}  // namespace nsb
