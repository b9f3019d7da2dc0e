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
//   * One warp per destination row.  Lane l works on batch row b = l % BT of
//     edge slot l / BT, so one gather instruction of the warp fetches the BT
//     contiguous floats of 32 / BT edges (for BT = 8: four 32-byte sectors in
//     one request) instead of one load per (edge, batch row).
//   * The warp loads 32 edges' columns and weights with one coalesced load
//     each and hands them to the (edge, batch) lanes with shuffles; all of a
//     batch's gathers are issued before its FMAs.
//   * Lane sums (edges l / BT, l / BT + 32/BT, ... in order) are reduced over
//     the lanes of a batch row with a fixed xor tree; lanes 0..BT-1 then apply
//     the pointwise update for their batch row.
#include <algorithm>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kThreads = 256;

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

template <int BT, bool UPDATE, typename W>
__global__ void __launch_bounds__(kThreads)
csr_batch_kernel(TickArgs t, View x, const int32_t* __restrict__ rowptr,
                 const int32_t* __restrict__ col, W weights, TickOut out, Out product) {
  constexpr int kEdgesPerStep = 32 / BT;
  const int lane = threadIdx.x & 31;
  const int b = lane % BT;
  const int slot = lane / BT;
  const int64_t neurons = t.neurons;
  const int64_t batch = t.batch;
  const int64_t b0 = static_cast<int64_t>(blockIdx.y) * BT;
  const bool active = b0 + b < batch;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const uint64_t pol = evict_first_policy();
  const float* __restrict__ xb = x.data + (active ? (b0 + b) * x.sb : 0);

  for (int64_t n = warp; n < neurons; n += n_warps) {
    const int64_t e0 = rowptr[n];
    const int64_t e1 = rowptr[n + 1];
    float acc = -0.0f;  // -0.0 is the exact additive identity
    for (int64_t e = e0; e < e1; e += 32) {
      const int count = static_cast<int>(e1 - e < 32 ? e1 - e : 32);
      int c = 0;
      float w = 0.0f;
      if (lane < count) {
        c = static_cast<int>(stream_load_u32(reinterpret_cast<const uint32_t*>(col + e + lane), pol));
        w = weights.one(e + lane);
      }
      float v[BT];
#pragma unroll
      for (int i = 0; i < BT; ++i) {  // gathers first: BT independent loads in flight
        const int k = i * kEdgesPerStep + slot;
        const int ck = __shfl_sync(0xffffffffu, c, k);
        v[i] = (k < count && active) ? __ldg(xb + static_cast<int64_t>(ck) * x.sn) : 0.0f;
      }
#pragma unroll
      for (int i = 0; i < BT; ++i) {
        const int k = i * kEdgesPerStep + slot;
        const float wk = __shfl_sync(0xffffffffu, w, k);
        if (k < count) acc = fmaf(wk, v[i], acc);
      }
    }
#pragma unroll
    for (int off = BT; off < 32; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane < BT && active) {
      if constexpr (UPDATE) {
        const Update r = advance_at(t, acc, b0 + b, n);
        out.s.put(b0 + b, n, r.s);
        out.d.put(b0 + b, n, r.d);
        out.a.put(b0 + b, n, r.a);
      } else {
        product.put(b0 + b, n, acc);
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

template <int BT, bool UPDATE, typename W>
cudaError_t launch_batch_variant(const TickArgs& t, const View& x, const Csr& csr, const W& weights,
                                 const TickOut& out, const Out& product, cudaStream_t stream) {
  auto kernel = csr_batch_kernel<BT, UPDATE, W>;
  static int occupancy[64] = {0};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  DeviceInfo info;
  err = device_info(&info);
  if (err != cudaSuccess) return err;
  int& occ = occupancy[device & 63];
  if (occ == 0) occ = resident_blocks(kernel);
  const int64_t rows_per_block = kThreads / 32;
  const int64_t needed = (t.neurons + rows_per_block - 1) / rows_per_block;
  const int64_t cap = static_cast<int64_t>(info.sm_count) * occ;
  const dim3 grid(static_cast<unsigned>(std::max<int64_t>(1, std::min(needed, cap))),
                  static_cast<unsigned>((t.batch + BT - 1) / BT));
  kernel<<<grid, kThreads, 0, stream>>>(t, x, csr.rowptr, csr.col, weights, out, product);
  return cudaGetLastError();
}

template <bool UPDATE, typename W>
cudaError_t dispatch_batch(const TickArgs& t, const View& x, const Csr& csr, const W& w,
                           const TickOut& out, const Out& product, cudaStream_t stream) {
  if (t.batch <= 2) return launch_batch_variant<2, UPDATE>(t, x, csr, w, out, product, stream);
  if (t.batch <= 4) return launch_batch_variant<4, UPDATE>(t, x, csr, w, out, product, stream);
  return launch_batch_variant<8, UPDATE>(t, x, csr, w, out, product, stream);
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
    return dispatch_batch<UPDATE>(t, x, csr, w, out, product, stream);
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

bool aligned(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) % bytes) == 0;
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
