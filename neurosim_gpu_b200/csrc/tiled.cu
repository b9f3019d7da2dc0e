// tiled.cu -- the matrix tick for B = 1 with the gathered state in shared memory.
//
// Why: at B = 1 every edge gathers one float s[col] at a random column.  Served
// from L2, those 4-byte gathers cost one L2 tag lookup each and cap the tick
// far below HBM bandwidth.  Here the columns are split into K blocks that fit
// in shared memory and every CTA streams its edges block by block, gathering
// from shared memory instead.
//
// Data layout (built once per weight version by neurosim_gpu_b200/tiled.py):
//   * CTA c owns destination rows [row_begin[c], row_begin[c+1]) (balanced by
//     edge count, one CTA per SM).
//   * A task is 32 of those rows x one column block k.  Lane i of the warp that
//     runs the task owns row task_rows[q][i]; its edges with col in block k
//     are stored at slots off + j*32 + i (j = 0..len-1), so each load of the
//     warp reads 32 consecutive slots.  Rows are sorted by piece length inside
//     (c, k) before grouping, so the padding to the task length is small.
//     Padding slots hold column index `block_cols` (a shared-memory zero) and
//     weight 0.
//   * col holds the column relative to its block.
// Pipeline per CTA (1024 threads):
//   * warp 31 (producer) copies column block k of s into buffer k % NBUF with a
//     TMA bulk copy (cp.async.bulk, completion on mbarrier full[b]); it reuses a
//     buffer after mbarrier empty[b] says all consumer warps left its block.
//   * warps 0..30 (consumers) take tasks in (block, sorted row group) order
//     from a shared counter, wait full[b] of the task's block, accumulate their
//     row's dot product sequentially and add it to jacc[k % NBUF][row].
//   * after all tasks, every thread applies the pointwise update to rows of the
//     CTA (j = jacc[0][row] + jacc[1][row]) and writes s', d', a'.
// Every mbarrier wait is bounded; on timeout the kernel records an error code
// in `status` and continues, so a fault in the pipeline never hangs the GPU.
#include <algorithm>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kTiledThreads = 1024;
constexpr int kConsumerWarps = kTiledThreads / 32 - 1;
constexpr int kProducerWarp = kTiledThreads / 32 - 1;
constexpr long long kWaitLimit = 1ll << 24;  // try_wait polls before giving up
constexpr int kTiledHeader = 64;             // mbarriers + task counter

// Error word used when the caller passes no status pointer.
__device__ int g_tiled_status;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

// Bounded wait for phase `parity` of `bar`; returns false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_addr(bar);
  for (long long i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void bulk_copy_to_smem(void* dst, const void* src, uint32_t bytes,
                                                  uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ int ld_stream_s32(const int* p, uint64_t pol) {
  int r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.s32 %0, [%1], %2;"
               : "=r"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t ld_stream_u32(const uint32_t* p, uint64_t pol) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t ld_stream_u16(const uint16_t* p, uint64_t pol) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;"
               : "=h"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t ld_stream_u8(const uint8_t* p, uint64_t pol) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u8 %0, [%1], %2;"
               : "=h"(r)
               : "l"(p), "l"(pol));
  return r;
}

// Per-slot weight readers of the tiled layout.  `slot` indexes the tiled
// arrays; `orig` is the edge's position in the original CSR (NVFP4 scales).
struct TiledF32 {
  const float* w;
  __device__ __forceinline__ float at(int64_t slot, uint64_t pol) const {
    return __uint_as_float(ld_stream_u32(reinterpret_cast<const uint32_t*>(w) + slot, pol));
  }
};
struct TiledF16 {
  const __half* w;
  __device__ __forceinline__ float at(int64_t slot, uint64_t pol) const {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(
        ld_stream_u16(reinterpret_cast<const uint16_t*>(w) + slot, pol))));
  }
};
struct TiledE4M3 {
  const uint8_t* codes;
  const float* global;
  __device__ __forceinline__ float at(int64_t slot, uint64_t pol) const {
    return __fmul_rn(e4m3_value(ld_stream_u8(codes + slot, pol)), __ldg(global));
  }
};

struct TiledArgs {
  const int32_t* row_begin;    // [C+1]
  const int32_t* task_ptr;     // [C*K+1]
  const int32_t* task_offset;  // [T]  first slot of the task
  const int32_t* task_len;     // [T]
  const int16_t* task_rows;    // [T*32] row relative to row_begin[c], -1 = empty lane
  const int32_t* task_orig;    // [T*32] NVFP4: CSR position of the lane's first edge
  const int32_t* col;          // [S] column relative to the block, block_cols = padding
  const void* weight;          // [S] (NVFP4: [S/2] packed codes)
  const uint8_t* scales;       // NVFP4 block scales of the original CSR
  const float* global_scale;
  int64_t n_scales;
  int32_t format;
  int32_t blocks;              // K
  int32_t block_cols;          // CB
  int32_t buffers;             // NBUF (1 or 2)
  int32_t max_rows;            // rows of the largest CTA range
  int64_t cols;                // length of the gathered source vector
};

template <typename W>
__device__ __forceinline__ float task_dot(const W& w, const int* __restrict__ col,
                                          const float* __restrict__ sb, int64_t base, int len,
                                          uint64_t pol) {
  float acc = -0.0f;
  int j = 0;
  for (; j + 8 <= len; j += 8) {
    int c[8];
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) c[u] = ld_stream_s32(col + base + (j + u) * 32, pol);
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = w.at(base + (j + u) * 32, pol);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = fmaf(v[u], sb[c[u]], acc);
  }
  for (; j < len; ++j) acc = fmaf(w.at(base + j * 32, pol), sb[ld_stream_s32(col + base + j * 32, pol)], acc);
  return acc;
}

__device__ __forceinline__ float task_dot_nvfp4(const TiledArgs& L, const int* __restrict__ col,
                                                const float* __restrict__ sb, int64_t base,
                                                int len, int orig, uint64_t pol) {
  const uint8_t* codes = static_cast<const uint8_t*>(L.weight);
  const float g = __ldg(L.global_scale);
  const int shift = (threadIdx.x & 1) * 4;  // slot parity = lane parity (base % 32 == 0)
  float acc = -0.0f;
  int64_t block = -1;
  float factor = 0.0f;
  for (int j = 0; j < len; ++j) {
    const int64_t slot = base + j * 32;
    const uint32_t code = (ld_stream_u8(codes + (slot >> 1), pol) >> shift) & 15u;
    const int64_t b = min(static_cast<int64_t>(orig + j) >> 4, L.n_scales - 1);
    if (b != block) {
      block = b;
      factor = __fmul_rn(e4m3_value(__ldg(L.scales + b)), g);
    }
    acc = fmaf(__fmul_rn(e2m1_value(code), factor), sb[ld_stream_s32(col + slot, pol)], acc);
  }
  return acc;
}

template <typename W>
__global__ void __launch_bounds__(kTiledThreads, 1)
tiled_tick_kernel(TiledArgs L, W w, TickArgs t, const float* __restrict__ x, TickOut out,
                  Out product, bool update, int* status) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  const int nbuf = L.buffers;
  const int cb_pad = L.block_cols + 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);            // [2]
  uint64_t* empty = full + 2;                                         // [2]
  int* next_task = reinterpret_cast<int*>(empty + 2);
  float* sbuf = reinterpret_cast<float*>(smem_raw + kTiledHeader);    // [nbuf][cb_pad]
  float* jacc = sbuf + nbuf * cb_pad;                                 // [nbuf][max_rows]
  int* st = status ? status : &g_tiled_status;

  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int row0 = L.row_begin[c];
  const int rows = L.row_begin[c + 1] - row0;
  const int K = L.blocks;
  const int task_first = L.task_ptr[c * K];
  const int task_count = L.task_ptr[(c + 1) * K] - task_first;

  for (int i = threadIdx.x; i < nbuf * L.max_rows; i += blockDim.x) jacc[i] = 0.0f;
  if (threadIdx.x < 4 * nbuf) sbuf[(threadIdx.x >> 2) * cb_pad + L.block_cols + (threadIdx.x & 3)] = 0.0f;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(full + b, 1);
      mbar_init(empty + b, kConsumerWarps);
    }
    *next_task = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kProducerWarp) {
    if (lane == 0) {
      for (int k = 0; k < K; ++k) {
        const int b = k % nbuf;
        const int use = k / nbuf;
        if (k >= nbuf && !mbar_wait(empty + b, (use - 1) & 1)) atomicExch(st, 1);
        fence_proxy_async_smem();
        const int first = k * L.block_cols;
        const int count = min(static_cast<int64_t>(L.block_cols), L.cols - first);
        const int bulk = count & ~3;  // 16-byte multiple, rest by plain stores
        float* dst = sbuf + b * cb_pad;
        for (int i = bulk; i < count; ++i) dst[i] = __ldg(x + first + i);
        mbar_arrive_expect_tx(full + b, static_cast<uint32_t>(bulk) * 4u);
        if (bulk > 0) bulk_copy_to_smem(dst, x + first, static_cast<uint32_t>(bulk) * 4u, full + b);
      }
      // Do not retire while a copy into this CTA's shared memory may be in flight.
      for (int k = max(0, K - nbuf); k < K; ++k)
        if (!mbar_wait(full + (k % nbuf), (k / nbuf) & 1)) atomicExch(st, 2);
    }
  } else {
    const uint64_t pol = evict_first_policy();
    int waited = -1;  // highest block whose full barrier this warp has observed
    int current = 0;  // block of the tasks this warp works on
    // Blocks are observed in order.  A warp leaves block `current` (arrives on
    // its empty barrier) only after it has seen that block's full barrier, so an
    // arrival can never be counted in the phase of an older block.
    auto observe = [&](int k) {
      if (waited < k) {
        if (!mbar_wait(full + (k % nbuf), (k / nbuf) & 1)) atomicExch(st, 3);
        waited = k;
      }
    };
    auto leave_until = [&](int k) {
      while (current < k) {
        observe(current);
        if (lane == 0 && current < K - nbuf) mbar_arrive(empty + (current % nbuf));
        ++current;
      }
    };
    while (true) {
      int q = 0;
      if (lane == 0) q = atomicAdd(next_task, 1);
      q = __shfl_sync(0xffffffffu, q, 0);
      if (q >= task_count) break;
      const int task = task_first + q;
      int k = current;  // tasks are ordered by block: find this task's block
      while (L.task_ptr[c * K + k + 1] <= task) ++k;
      leave_until(k);
      observe(k);
      __syncwarp();
      const int row = L.task_rows[static_cast<int64_t>(task) * 32 + lane];
      const int64_t base = static_cast<int64_t>(L.task_offset[task]) + lane;
      const int len = L.task_len[task];
      const float* sb = sbuf + (k % nbuf) * cb_pad;
      float acc;
      if (L.format == NSB_WEIGHT_NVFP4) {
        acc = task_dot_nvfp4(L, L.col, sb, base, len,
                             L.task_orig[static_cast<int64_t>(task) * 32 + lane], pol);
      } else {
        acc = task_dot(w, L.col, sb, base, len, pol);
      }
      if (row >= 0) jacc[(k % nbuf) * L.max_rows + row] += acc;
    }
    leave_until(K);  // leave every remaining block (arrivals the producer may need)
  }
  __syncthreads();

  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const float j = nbuf == 2 ? jacc[r] + jacc[L.max_rows + r] : jacc[r];
    const int64_t n = row0 + r;
    if (update) {
      const Update u = advance_at(t, j, 0, n);
      out.s.put(0, n, u.s);
      out.d.put(0, n, u.d);
      out.a.put(0, n, u.a);
    } else {
      product.put(0, n, j);
    }
  }
}

template <typename W>
cudaError_t launch_tiled_variant(const TiledArgs& L, const W& w, const TickArgs& t,
                                 const float* x, const TickOut& out, const Out& product,
                                 bool update, int* status, int ctas, cudaStream_t stream) {
  const size_t smem = tiled_smem_bytes(L.block_cols, L.max_rows, L.buffers);
  auto kernel = tiled_tick_kernel<W>;
  static int configured[64] = {0};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  if (configured[device & 63] < static_cast<int>(smem)) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(smem));
    if (err != cudaSuccess) return err;
    configured[device & 63] = static_cast<int>(smem);
  }
  kernel<<<ctas, kTiledThreads, smem, stream>>>(L, w, t, x, out, product, update, status);
  return cudaGetLastError();
}

}  // namespace

size_t tiled_smem_bytes(int block_cols, int max_rows, int buffers) {
  return kTiledHeader + static_cast<size_t>(buffers) * (block_cols + 4) * 4 +
         static_cast<size_t>(buffers) * max_rows * 4;
}

cudaError_t launch_tiled(const nsb_tiled_layout& layout, const TickArgs& t, const float* x,
                         bool update, const TickOut& out, const Out& product, int* status,
                         cudaStream_t stream) {
  TiledArgs L;
  L.row_begin = layout.row_begin;
  L.task_ptr = layout.task_ptr;
  L.task_offset = layout.task_offset;
  L.task_len = layout.task_len;
  L.task_rows = layout.task_rows;
  L.task_orig = layout.task_orig;
  L.col = layout.col;
  L.weight = layout.weight;
  L.scales = layout.block_scales;
  L.global_scale = layout.global_scale;
  L.n_scales = layout.n_block_scales;
  L.format = layout.format;
  L.blocks = layout.blocks;
  L.block_cols = layout.block_cols;
  L.buffers = layout.buffers;
  L.max_rows = layout.max_rows;
  L.cols = layout.cols;
  const int ctas = layout.ctas;
  switch (layout.format) {
    case NSB_WEIGHT_F16:
      return launch_tiled_variant(L, TiledF16{static_cast<const __half*>(layout.weight)}, t, x,
                                  out, product, update, status, ctas, stream);
    case NSB_WEIGHT_E4M3:
      return launch_tiled_variant(L, TiledE4M3{static_cast<const uint8_t*>(layout.weight),
                                               layout.global_scale},
                                  t, x, out, product, update, status, ctas, stream);
    case NSB_WEIGHT_NVFP4:
      return launch_tiled_variant(L, TiledF32{nullptr}, t, x, out, product, update, status, ctas,
                                  stream);
    default:
      return launch_tiled_variant(L, TiledF32{static_cast<const float*>(layout.weight)}, t, x,
                                  out, product, update, status, ctas, stream);
  }
}

}  // namespace nsb
