// cluster.cu -- the matrix tick of a small graph on one thread-block cluster.
//
// For graphs whose state vector and edges fit in the shared memory of one
// cluster (N = 4,096 / M = 65k: about 135 KB per CTA), T ticks run inside one
// cluster of kClusterCtas CTAs with no global-memory traffic between ticks:
//   * every CTA keeps the WHOLE state vector s, double-buffered, and its own
//     rows' edges (columns and weights decoded to float32), d, a, parameters
//     and drives in shared memory;
//   * CTA c owns rows [c*R, (c+1)*R), R = ceil(N / kClusterCtas) rounded up to
//     a multiple of 32; thread i of the CTA owns rows i, i + kClusterThreads,
//     ...; each warp's 32 rows are stored interleaved (slot k of the row of
//     lane l at warp_base + 32*k + l, warp_base from the warps' largest
//     degrees), so the edge reads of a warp are conflict-free;
//   * a thread sums its row sequentially in CSR order, applies the pointwise
//     update and stores the new s of the row into the next state buffer of
//     EVERY CTA of the cluster (distributed shared memory);
//   * one cluster barrier per tick (arrive.release / wait.acquire) orders those
//     stores before the next tick's reads, and all reads of the current buffer
//     before it is overwritten one tick later.
// After T ticks each CTA writes its rows' s, d, a to the outputs.  A rollout
// (drive tick stride > 0 or a history) reads tick k's drive from global memory
// k strides on and writes every tick's new s of its rows to history row k.
#include <cooperative_groups.h>

#include <algorithm>
#include <vector>

#include "nsb_launch.h"

namespace cg = cooperative_groups;

namespace nsb {
namespace {

constexpr int kClusterCtas = 8;
constexpr int kClusterThreads = 512;

struct ClusterArgs {
  const int32_t* rowptr;   // [N+1]
  const int32_t* col;      // [M]
  int64_t rows_per_cta;    // R, a multiple of 32
  int64_t max_slots;       // interleaved edge slots one CTA may hold
  int64_t n_pad;           // N rounded up to 4
};

__device__ __forceinline__ int64_t clamp_rows(int64_t x, int64_t limit) {
  return x < limit ? x : limit;
}

__device__ __forceinline__ int degree(const int32_t* rowptr, int64_t row, int64_t n) {
  return row < n ? __ldg(rowptr + row + 1) - __ldg(rowptr + row) : 0;
}

template <typename W>
__global__ void __cluster_dims__(kClusterCtas, 1, 1) __launch_bounds__(kClusterThreads, 1)
cluster_tick_kernel(ClusterArgs A, W weights, TickArgs t, TickOut out, int ticks, int* status,
                    Out history) {
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int lane = threadIdx.x & 31;
  const int64_t n = t.neurons;
  const int64_t R = A.rows_per_cta;
  const int warps = static_cast<int>(R >> 5);

  // Dynamic shared memory: need[kClusterCtas] (int64), warp_base[warps + 1]
  // padded to 4 ints, then the float arrays (cluster_smem_bytes).
  extern __shared__ __align__(16) unsigned char smem_raw[];
  int64_t* need = reinterpret_cast<int64_t*>(smem_raw);
  int* warp_base = reinterpret_cast<int*>(need + kClusterCtas);
  if (threadIdx.x < kClusterCtas) need[threadIdx.x] = 0;
  __syncthreads();
  // Every CTA computes every CTA's slot count from the same rowptr, so they
  // all take the same decision below (before any cluster barrier).
  for (int64_t i = threadIdx.x; i < kClusterCtas * R; i += blockDim.x) {
    const int widest = __reduce_max_sync(0xffffffffu, degree(A.rowptr, i, n));
    const int c = static_cast<int>(i / R);
    if (lane == 0) {
      atomicAdd(reinterpret_cast<unsigned long long*>(&need[c]),
                static_cast<unsigned long long>(32 * widest));
      if (c == rank) warp_base[(i - c * R) >> 5] = widest;
    }
  }
  __syncthreads();
  for (int c = 0; c < kClusterCtas; ++c) {
    if (need[c] > A.max_slots) {
      if (status && threadIdx.x == 0) atomicExch(status, 7);
      return;
    }
  }
  if (threadIdx.x == 0) {
    int running = 0;
    for (int w = 0; w < warps; ++w) {
      const int widest = warp_base[w];
      warp_base[w] = running;
      running += 32 * widest;
    }
    warp_base[warps] = running;
  }

  float* smem = reinterpret_cast<float*>(warp_base + ((warps + 4) & ~3));
  float* d = smem + 2 * A.n_pad;  // smem[0, 2*n_pad): the two state buffers
  float* a = d + R;
  float* prm = a + R;  // [6][R]
  float* uu = prm + 6 * R;
  float* vv = uu + R;
  int* dg = reinterpret_cast<int*>(vv + R);  // [R] row degrees
  int* cc = dg + R;                          // [max_slots]
  float* ww = reinterpret_cast<float*>(cc + A.max_slots);

  const int64_t row0 = clamp_rows(rank * R, n);
  const int64_t rows = clamp_rows(R, n - row0);

  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) smem[i] = t.s.at(0, i);
  __syncthreads();  // warp_base complete
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    const int64_t row = row0 + r;
    d[r] = t.d.at(0, row);
    a[r] = t.a.at(0, row);
    for (int k = 0; k < 6; ++k) prm[k * R + r] = t.p.at(k, row);
    uu[r] = t.u.at(0, row);
    vv[r] = t.v.at(0, row);
    const int64_t e0 = __ldg(A.rowptr + row);
    const int deg = __ldg(A.rowptr + row + 1) - static_cast<int>(e0);
    dg[r] = deg;
    const int base = warp_base[r >> 5] + lane;
    for (int k = 0; k < deg; ++k) {
      cc[base + 32 * k] = __ldg(A.col + e0 + k);
      ww[base + 32 * k] = weights.one(e0 + k);
    }
  }
  // Every CTA has its own copy of s; the first remote stores go to the other
  // buffer, so the cluster only has to start together.
  cluster.sync();

  for (int tick = 0; tick < ticks; ++tick) {
    const float* sc = smem + (tick & 1) * A.n_pad;
    float* next = smem + ((tick + 1) & 1) * A.n_pad;
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
      const int w = static_cast<int>(r >> 5);
      const int base = warp_base[w] + lane;
      const int deg = (warp_base[w + 1] - warp_base[w]) >> 5;  // the warp's widest row
      const int mine = dg[r];
      float j = -0.0f;  // -0.0 is the exact additive identity
      int k = 0;
      // Four slots per step, all loads first (slots below the warp's widest
      // row are allocated), then the multiply-adds in CSR order.
      for (; k + 4 <= deg; k += 4) {
        int c[4];
        float w[4], x[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          c[q] = cc[base + 32 * (k + q)];
          w[q] = ww[base + 32 * (k + q)];
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) x[q] = sc[k + q < mine ? c[q] : 0];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (k + q < mine) j = fmaf(w[q], x[q], j);
      }
      for (; k < mine; ++k) j = fmaf(ww[base + 32 * k], sc[cc[base + 32 * k]], j);
      const float u = t.u.sb ? t.u.at(tick, row0 + r) : uu[r];  // batch stride = tick stride
      const Update q = advance(j, sc[row0 + r], d[r], a[r], u, vv[r], prm[r], prm[R + r],
                               prm[2 * R + r], prm[3 * R + r], prm[4 * R + r], prm[5 * R + r]);
      d[r] = q.d;
      a[r] = q.a;
      if (history.data) history.put(tick, row0 + r, q.s);
#pragma unroll
      for (int peer = 0; peer < kClusterCtas; ++peer)
        cluster.map_shared_rank(next, peer)[row0 + r] = q.s;
    }
    cluster.sync();
  }

  const float* final_s = smem + (ticks & 1) * A.n_pad;
  for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    const int64_t row = row0 + r;
    out.s.put(0, row, final_s[row]);
    out.d.put(0, row, d[r]);
    out.a.put(0, row, a[r]);
  }
}

template <typename W>
cudaError_t launch_cluster_variant(const ClusterArgs& A, const W& w, const TickArgs& t,
                                   const TickOut& out, int ticks, size_t smem, int* status,
                                   const Out& history, cudaStream_t stream) {
  auto kernel = cluster_tick_kernel<W>;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
  if (err != cudaSuccess) return err;
  kernel<<<kClusterCtas, kClusterThreads, smem, stream>>>(A, w, t, out, ticks, status, history);
  return cudaGetLastError();
}

int64_t rows_per_cta(int64_t neurons) {
  const int64_t r = (neurons + kClusterCtas - 1) / kClusterCtas;
  return (r + 31) & ~int64_t{31};
}

}  // namespace

int64_t cluster_slots(int64_t neurons, const int32_t* host_rowptr) {
  const int64_t R = rows_per_cta(neurons);
  int64_t most = 0;
  for (int c = 0; c < kClusterCtas; ++c) {
    int64_t slots = 0;
    for (int64_t w0 = c * R; w0 < (c + 1) * R && w0 < neurons; w0 += 32) {
      int widest = 0;
      for (int64_t row = w0; row < w0 + 32 && row < neurons; ++row)
        widest = std::max(widest, host_rowptr[row + 1] - host_rowptr[row]);
      slots += 32 * int64_t{widest};
    }
    most = std::max(most, slots);
  }
  return most;
}

size_t cluster_smem_bytes(int64_t neurons, int64_t max_slots) {
  const int64_t R = rows_per_cta(neurons);
  const int64_t n_pad = (neurons + 3) & ~int64_t{3};
  const int64_t head = kClusterCtas * 8 + ((R / 32 + 4) & ~int64_t{3}) * 4;
  return static_cast<size_t>(head + 2 * n_pad * 4 + R * 11 * 4 + max_slots * 8);
}

cudaError_t launch_cluster(const TickArgs& tick, const Csr& csr, int64_t max_slots, int ticks,
                           const TickOut& out, int* status, cudaStream_t stream,
                           int64_t drive_tick_stride, const Out& history) {
  TickArgs t = tick;
  t.u.sb = t.u.data ? drive_tick_stride : 0;  // B = 1: the batch stride is the tick stride
  const size_t smem = cluster_smem_bytes(t.neurons, max_slots);
  ClusterArgs A;
  A.rowptr = csr.rowptr;
  A.col = csr.col;
  A.rows_per_cta = rows_per_cta(t.neurons);
  A.max_slots = max_slots;
  A.n_pad = (t.neurons + 3) & ~int64_t{3};
  switch (csr.format) {
    case NSB_WEIGHT_F16:
      return launch_cluster_variant(A, WeightsF16{static_cast<const __half*>(csr.weight)}, t, out,
                                    ticks, smem, status, history, stream);
    case NSB_WEIGHT_E4M3:
      return launch_cluster_variant(
          A, WeightsE4M3{static_cast<const uint8_t*>(csr.weight), csr.global_scale}, t, out, ticks,
          smem, status, history, stream);
    case NSB_WEIGHT_NVFP4:
      return launch_cluster_variant(
          A, WeightsNVFP4{static_cast<const uint8_t*>(csr.weight), csr.block_scales,
                          csr.global_scale},
          t, out, ticks, smem, status, history, stream);
    default:
      return launch_cluster_variant(A, WeightsF32{static_cast<const float*>(csr.weight)}, t, out,
                                    ticks, smem, status, history, stream);
  }
}

}  // namespace nsb
