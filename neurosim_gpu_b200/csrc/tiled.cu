// tiled.cu -- the matrix tick for B = 1 with the gathered state in shared memory.
//
// Why: at B = 1 every edge gathers one float s[col] at a random column.  Served
// from L2, those 4-byte gathers cost one L2 tag lookup each and cap the tick
// far below HBM bandwidth.  Here the gathered columns are split into blocks
// that fit in one CTA's shared memory, and each CTA streams the edges of one
// column block (a "stage": that block x a range of destination rows), so the
// gathers hit shared memory and each block of the state is staged once per
// tick per CTA that needs it.
//
// Data layout (built once per weight version by neurosim_gpu_b200/tiled.py):
//   * CTA c runs stages stage_ptr[c] .. stage_ptr[c+1]-1 (normally one).
//   * A segment is 32 rows x the stage's block: lane i owns one row, and its
//     edges in the block form a contiguous run of its CSR row (the "piece").
//     A segment has C chunks of K slots per lane (K = 4, 8, or 16 for E4M3 /
//     NVFP4; one K per layout); chunk c of lane i holds the lane's edges
//     Kc..Kc+K-1 at slots first + 32Kc + Ki + (0..K-1), so one load of the
//     K 16-bit columns (8, 16 or 32 bytes) and one vector load of the
//     weights serve K edges, and a warp's loads cover 32K consecutive slots.
//     A lane sums its piece in CSR order whatever K is.  Padding slots hold column
//     `block_cols` (a shared-memory zero) and weight 0.  A task is one
//     segment (lane i's row: task_rows[32q+i] & 0x0FFFFFFF), or, for fp32,
//     several equal segments one after the other (segment k's rows: row group
//     tasks[q].w + k of task_rows), so short pieces do not cost one task
//     hand-out per 32 of them.
//   * NVFP4: the nibble of slot s is in byte s/2 (even slot low).  Edge j of a
//     lane sits at CSR position o + j and takes the E4M3 scale of CSR block
//     (o + j) / 16.  Per task, scale_pairs[first pair + 32b + i] = (scale of
//     block o/16 + b) | (scale of block o/16 + b + 1) << 8, so a chunk needs one
//     2-byte load for both scales it can touch; the lane's phase o % 16 sits in
//     bits 28..31 of its task_rows word.
// One launch runs `ticks` ticks (a cooperative launch, one CTA per SM):
//   1. warp 31 (producer) copies the block of each stage into a shared-memory
//      buffer with a TMA bulk copy (cp.async.bulk, completion on mbarrier
//      full[b]); with two buffers it reuses one after mbarrier empty[b] says all
//      consumer warps left its stage.
//   2. warps 0..30 (consumers) take tasks (sub-tasks: one split of 32 rows'
//      pieces) from a shared counter.  Each warp
//      keeps a ring of D chunks in registers: the loads of a chunk are issued D
//      chunks before it is used, across task and stage boundaries, so a warp
//      always has D chunks of edges in flight (also while the state block is
//      still being staged).  A lane's sum over its split of the piece
//      (sequential, CSR order) is stored to part[block][split][row].
//   3. grid barrier; every CTA takes rows [c*R/C, (c+1)*R/C), adds their sums
//      in (block, split) order (clearing part for the next tick), applies the
//      pointwise update and writes s', d', a' (and, for a rollout, s' into the
//      history row of the tick; tick k's drive is read k drive strides on).
//   4. for the next tick (in place on the outputs): back to 1; the producer
//      waits at a grid barrier (every CTA's update done) before it stages the
//      new state, while the consumers already load the next tick's edges.
// Every wait (mbarrier or grid barrier) is bounded; on timeout the kernel
// records an error code in `status` and continues, so a fault in the pipeline
// never hangs the GPU.
#include <algorithm>
#include <type_traits>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kTiledThreads = 1024;
constexpr int kConsumerWarps = kTiledThreads / 32 - 1;
constexpr int kProducerWarp = kTiledThreads / 32 - 1;
constexpr long long kWaitLimit = 1ll << 24;  // try_wait polls before giving up
constexpr long long kGridWaitLimit = 1ll << 24;  // polls of the grid barrier
constexpr int kTiledHeader = 64;             // mbarriers + task counter
// L2 prefetch of task data by the producer warp: bytes of tasks a CTA keeps
// prefetched beyond the hand-out counter.  Only the narrower weight formats
// use it: an fp32 tick streams more bytes than L2 holds, and prefetched lines
// were evicted before use (measured: 43.9 us without, 46-51 us with).
constexpr int kPrefetchBudget = 128 << 10;
constexpr uint32_t kRowMask = 0x0FFFFFFFu;   // task_rows: row bits; kRowMask = padding lane

// Tag of a chunk in a consumer's ring (one 32-bit word per lane).
constexpr uint32_t kTagValid = 1u;
constexpr uint32_t kTagLast = 2u;   // last chunk of its task
constexpr int kTagPhase = 2;        // NVFP4: (phase + K c) % 16, 4 bits
constexpr int kTagStage = 6;        // CTA-local stage, 16 bits
constexpr int kTagSplit = 22;       // split of the sub-task, 10 bits

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

// Streaming loads: read once per tick, no L1 allocation, evict-first in L2.
__device__ __forceinline__ uint32_t ld_stream_u16(const void* p, uint64_t pol) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u16 %0, [%1], %2;"
               : "=h"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint32_t ld_stream_u32(const void* p, uint64_t pol) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(r)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint2 ld_stream_v2(const void* p, uint64_t pol) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0,%1}, [%2], %3;"
               : "=r"(r.x), "=r"(r.y)
               : "l"(p), "l"(pol));
  return r;
}

__device__ __forceinline__ uint4 ld_stream_v4(const void* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}

// Bulk prefetch of [p, p + bytes) into L2 (16-byte aligned, multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Two E4M3 codes (low byte first) -> two floats, exact (every E4M3 value is
// an f16 value).  Hardware conversion on sm_100a.
__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two) {
  uint32_t h;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, lo;\n\t}"
      : "=r"(h)
      : "r"(two));
  return __half22float2(*reinterpret_cast<__half2*>(&h));
}

// Four E2M1 codes (nibbles, lowest first) -> four floats, exact.
__device__ __forceinline__ void e2m1x4_to_float(uint32_t four, float (&v)[4]) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\tmov.b32 {b0, b1, b2, b3}, %2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\tcvt.rn.f16x2.e2m1x2 %1, b1;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(four));
  const float2 a = __half22float2(*reinterpret_cast<__half2*>(&h0));
  const float2 b = __half22float2(*reinterpret_cast<__half2*>(&h1));
  v[0] = a.x;
  v[1] = a.y;
  v[2] = b.x;
  v[3] = b.y;
}

// 256-bit streaming load (eight 32-bit words).
struct Words8 {
  uint32_t v[8];
};

__device__ __forceinline__ Words8 ld_stream_v8(const void* p, uint64_t pol) {
  Words8 r;
  asm volatile(
      "ld.global.nc.L1::no_allocate.L2::cache_hint.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
      : "=r"(r.v[0]), "=r"(r.v[1]), "=r"(r.v[2]), "=r"(r.v[3]), "=r"(r.v[4]), "=r"(r.v[5]),
        "=r"(r.v[6]), "=r"(r.v[7])
      : "l"(p), "l"(pol));
  return r;
}

// The K 16-bit block-relative columns of one lane's chunk: one 8-byte (K = 4)
// or 16-byte (K = 8) load.
template <int K>
struct ChunkCols;

template <>
struct ChunkCols<4> {
  using Raw = uint2;
  static __device__ __forceinline__ Raw load(const uint16_t* col, int64_t slot, uint64_t pol) {
    return ld_stream_v2(col + slot, pol);
  }
  static __device__ __forceinline__ uint32_t at(const Raw& r, int e) {
    const uint32_t word = e < 2 ? r.x : r.y;
    return (e & 1) ? word >> 16 : word & 0xFFFFu;
  }
};

template <>
struct ChunkCols<8> {
  using Raw = uint4;
  static __device__ __forceinline__ Raw load(const uint16_t* col, int64_t slot, uint64_t pol) {
    return ld_stream_v4(col + slot, pol);
  }
  static __device__ __forceinline__ uint32_t at(const Raw& r, int e) {
    const uint32_t word = e < 2 ? r.x : e < 4 ? r.y : e < 6 ? r.z : r.w;
    return (e & 1) ? word >> 16 : word & 0xFFFFu;
  }
};

template <>
struct ChunkCols<16> {
  using Raw = Words8;
  static __device__ __forceinline__ Raw load(const uint16_t* col, int64_t slot, uint64_t pol) {
    return ld_stream_v8(col + slot, pol);
  }
  static __device__ __forceinline__ uint32_t at(const Raw& r, int e) {
    const uint32_t word = r.v[e >> 1];
    return (e & 1) ? word >> 16 : word & 0xFFFFu;
  }
};

// Chunk readers, for K slots per lane (one lane's chunk): load(slot,
// scale_entry) fetches the K weights; decode() turns them into K float32
// weights, equal bit for bit to the reference quantizer's dequantized values
// (precision.py:102-109): fp8 -> e4m3(code) * g, nvfp4 -> e2m1(code) *
// (e4m3(block scale) * g).
template <int K>
struct ChunkF32 {
  static constexpr int kSlots = K;
  static constexpr bool kF32 = true;
  using Raw = typename std::conditional<K == 4, uint4, Words8>::type;
  const float* w;
  __device__ __forceinline__ void prefetch(int first, int chunks, int, int) const {
    prefetch_l2(w + first, static_cast<uint32_t>(chunks) * 32u * K * 4u);
  }
  __device__ __forceinline__ void set_scale(float) {}
  __device__ __forceinline__ Raw load(int64_t slot, int64_t, uint64_t pol) const {
    if constexpr (K == 4) return ld_stream_v4(w + slot, pol);
    else return ld_stream_v8(w + slot, pol);
  }
  __device__ __forceinline__ void decode(const Raw& r, uint32_t, float (&v)[K]) const {
    if constexpr (K == 4) {
      v[0] = __uint_as_float(r.x);
      v[1] = __uint_as_float(r.y);
      v[2] = __uint_as_float(r.z);
      v[3] = __uint_as_float(r.w);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(r.v[e]);
    }
  }
};

template <int K>
struct ChunkF16 {
  static constexpr int kSlots = K;
  static constexpr bool kF32 = false;
  using Raw = typename std::conditional<K == 4, uint2,
                                       typename std::conditional<K == 8, uint4, Words8>::type>::type;
  const __half* w;
  __device__ __forceinline__ void prefetch(int first, int chunks, int, int) const {
    prefetch_l2(w + first, static_cast<uint32_t>(chunks) * 32u * K * 2u);
  }
  __device__ __forceinline__ void set_scale(float) {}
  __device__ __forceinline__ Raw load(int64_t slot, int64_t, uint64_t pol) const {
    if constexpr (K == 4) return ld_stream_v2(w + slot, pol);
    else if constexpr (K == 8) return ld_stream_v4(w + slot, pol);
    else return ld_stream_v8(w + slot, pol);
  }
  __device__ __forceinline__ void decode(const Raw& r, uint32_t, float (&v)[K]) const {
    const uint32_t* words = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < K / 2; ++i) {
      const float2 h = __half22float2(*reinterpret_cast<const __half2*>(words + i));
      v[2 * i] = h.x;
      v[2 * i + 1] = h.y;
    }
  }
};

template <int K>
struct ChunkE4M3 {
  static constexpr int kSlots = K;
  static constexpr bool kF32 = false;
  using Raw = typename std::conditional<K == 4, uint32_t,
                                       typename std::conditional<K == 8, uint2, uint4>::type>::type;
  const uint8_t* codes;
  float g;
  __device__ __forceinline__ void prefetch(int first, int chunks, int, int) const {
    prefetch_l2(codes + first, static_cast<uint32_t>(chunks) * 32u * K);
  }
  __device__ __forceinline__ void set_scale(float s) { g = s; }
  __device__ __forceinline__ Raw load(int64_t slot, int64_t, uint64_t pol) const {
    if constexpr (K == 4) return ld_stream_u32(codes + slot, pol);
    else if constexpr (K == 8) return ld_stream_v2(codes + slot, pol);
    else return ld_stream_v4(codes + slot, pol);
  }
  __device__ __forceinline__ void decode(const Raw& r, uint32_t, float (&v)[K]) const {
    const uint32_t* words = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < K / 4; ++i) {
      const float2 a = e4m3x2_to_float2(words[i] & 0xFFFFu);
      const float2 b = e4m3x2_to_float2(words[i] >> 16);
      v[4 * i] = __fmul_rn(a.x, g);
      v[4 * i + 1] = __fmul_rn(a.y, g);
      v[4 * i + 2] = __fmul_rn(b.x, g);
      v[4 * i + 3] = __fmul_rn(b.y, g);
    }
  }
};

template <int K>
struct ChunkNVFP4 {
  static constexpr int kSlots = K;
  static constexpr bool kF32 = false;
  // K = 4: four codes (low 16 bits) | scale pair << 16; K = 8: eight codes,
  // scale pair; K = 16: sixteen codes (x, y), scale pair (z).
  using Raw = typename std::conditional<K == 4, uint32_t,
                                       typename std::conditional<K == 8, uint2, uint4>::type>::type;
  const uint8_t* codes;
  const uint16_t* pairs;
  float g;
  // Codes and the scale-table rows a split of C chunks starting at chunk c0
  // of the lanes' pieces reads: rows (K c0) / 16 .. (K (c0 + C) + 15 - K) / 16.
  __device__ __forceinline__ void prefetch(int first, int chunks, int entry, int c0) const {
    prefetch_l2(codes + (first >> 1), static_cast<uint32_t>(chunks) * 16u * K);
    const int r0 = (K * c0) >> 4;
    const int r1 = (K * (c0 + chunks) + 15 - K) >> 4;
    prefetch_l2(pairs + entry + r0 * 32, static_cast<uint32_t>(r1 - r0 + 1) * 64u);
  }
  __device__ __forceinline__ void set_scale(float s) { g = s; }
  __device__ __forceinline__ Raw load(int64_t slot, int64_t entry, uint64_t pol) const {
    if constexpr (K == 4) {
      return ld_stream_u16(codes + (slot >> 1), pol) | (static_cast<uint32_t>(__ldg(pairs + entry)) << 16);
    } else if constexpr (K == 8) {
      return make_uint2(ld_stream_u32(codes + (slot >> 1), pol), __ldg(pairs + entry));
    } else {
      const uint2 c = ld_stream_v2(codes + (slot >> 1), pol);
      return make_uint4(c.x, c.y, __ldg(pairs + entry), 0u);
    }
  }
  __device__ __forceinline__ void decode(const Raw& r, uint32_t tag, float (&v)[K]) const {
    uint32_t codes4[K / 4];
    uint32_t pair;
    if constexpr (K == 4) {
      codes4[0] = r & 0xFFFFu;
      pair = r >> 16;
    } else if constexpr (K == 8) {
      codes4[0] = r.x & 0xFFFFu;
      codes4[1] = r.x >> 16;
      pair = r.y;
    } else {
      codes4[0] = r.x & 0xFFFFu;
      codes4[1] = r.x >> 16;
      codes4[2] = r.y & 0xFFFFu;
      codes4[3] = r.y >> 16;
      pair = r.z;
    }
    const float2 scale = e4m3x2_to_float2(pair);
    const float f0 = __fmul_rn(scale.x, g), f1 = __fmul_rn(scale.y, g);
    const int phase = (tag >> kTagPhase) & 15;  // edge e is in the next block iff phase + e >= 16
#pragma unroll
    for (int i = 0; i < K / 4; ++i) {
      float q[4];
      e2m1x4_to_float(codes4[i], q);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        v[4 * i + e] = __fmul_rn(q[e], phase + 4 * i + e >= 16 ? f1 : f0);
    }
  }
};

struct TiledArgs {
  const int32_t* stage_ptr;    // [C+1]
  const int32_t* stage_block;  // [stages]
  const int32_t* task_ptr;     // [C+1]
  const int4* tasks;           // [T]: first slot, chunks, stage | split << 16 | segment << 26,
                               //      NVFP4: first scale pair, else: first row group
  const int32_t* task_rows;    // NVFP4 [T*32]: row | phase << 28; else [groups*32]: row
  const uint16_t* col;         // [S] column relative to the block, block_cols = padding
  const float* global_scale;   // E4M3 / NVFP4: one float
  float* part;                 // workspace: [blocks][splits][rows] row sums (zero between launches)
  unsigned long long* barrier; // workspace: grid-barrier arrival counter
  int32_t block_cols;          // CB
  int32_t buffers;             // NBUF (1 or 2)
  int32_t prefetch_ahead;      // tasks prefetched beyond the hand-out counter
  int32_t prefetch_first;      // tasks of the next tick's first round prefetched (0 or warps)
  int32_t splits;              // sub-task planes per block
  int32_t split_chunks;        // chunks of one sub-task
  int32_t stage_rows;          // staged update: rows per chunk (a multiple of 4; 0: loads)
  int64_t rows;                // destination rows
  int64_t cols;                // length of the gathered source vector
};

__device__ __forceinline__ unsigned long long ld_acquire_gpu(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of a cooperative launch over a monotonic 64-bit arrival
// counter, for one thread per CTA (after a __syncthreads that orders the CTA's
// writes before it): the CTA whose arrival is number a (0-based) waits until
// the counter reaches the next multiple of the grid size above a.  Nothing is
// reset, so the critical path is one atomic and the pollers' next read.
// Every launch that uses a workspace has the same grid size and passes every
// barrier, so the counter is a multiple of the grid size between launches.
// The arrival is a release (cumulative over the CTA's writes ordered before
// it by the __syncthreads) and the poll an acquire, so no full fence is needed
// on either side: a trailing fence also waited for this thread's own L2
// prefetches in flight (166k / 25M: 34.85 -> 34.15 us per tick).
// The wait is bounded: on timeout it records code 4.
__device__ void grid_arrive_wait(unsigned long long* count, int* st) {
  unsigned long long arrival;
  asm volatile("atom.add.release.gpu.global.u64 %0, [%1], 1;" : "=l"(arrival) : "l"(count) : "memory");
  const unsigned long long target = (arrival / gridDim.x + 1) * gridDim.x;
  long long polls = 0;
  while (ld_acquire_gpu(count) < target) {
    if (++polls > (1 << 16)) {
      if (polls > kGridWaitLimit) {
        atomicExch(st, 4);
        break;
      }
      __nanosleep(256);
    }
  }
}

// The same barrier for the whole CTA.
__device__ void grid_barrier(unsigned long long* count, int* st) {
  __syncthreads();
  if (threadIdx.x == 0) grid_arrive_wait(count, st);
  __syncthreads();
}

// The peer exchange of a row-sharded run (world == 0: none).
struct Peers {
  int32_t world, rank;
  int64_t row_offset;
  float* gathered[NSB_MAX_PEERS][2];
  unsigned long long* counters[NSB_MAX_PEERS];
  unsigned long long epoch;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// End-of-tick barrier across ranks, for one thread per CTA after a
// __syncthreads that follows the CTA's peer stores and a system-scope fence by
// that thread: every CTA counts its arrival on the rank's local counter, and
// the CTA that arrives last (its atomic follows every other CTA's arrival,
// each made after that CTA's fence) fences and adds one to every rank's
// counter.  Every CTA then waits until its rank's counter shows all ranks'
// arrivals for this tick; none waits on the local counter, so the signal
// leaves as soon as the rank's last CTA is done.  The local counter still
// grows by the grid size per tick.  Bounded: on timeout it records code 6.
__device__ void peer_barrier(const Peers& px, unsigned long long* local, int tick, int* st) {
  const unsigned long long arrival = atomicAdd(local, 1ull);
  if (arrival % gridDim.x == gridDim.x - 1) {
    __threadfence_system();
    for (int p = 0; p < px.world; ++p) atomicAdd_system(px.counters[p], 1ull);
  }
  const unsigned long long target =
      static_cast<unsigned long long>(px.world) * (px.epoch + static_cast<unsigned long long>(tick) + 1);
  long long polls = 0;
  while (ld_acquire_sys(px.counters[px.rank]) < target) {
    if (++polls > (1 << 16)) {
      if (polls > kGridWaitLimit) {
        atomicExch(st, 6);
        break;
      }
      __nanosleep(256);
    }
  }
}

// X: the row-sharded variant with the peer exchange (nsb_dendritic_run_tiled_peers);
// the single-GPU instantiation carries none of its code.
// G: the gated, accumulating propagate-only launch of the hybrid PELS tick.
template <typename W, int D, bool X, bool G>
__global__ void __launch_bounds__(kTiledThreads, 1)
tiled_tick_kernel(TiledArgs L, W weights, TickArgs t, const float* __restrict__ x0, TickOut out,
                  Out product, bool update, int ticks, int* status, Peers px,
                  const unsigned long long* gate_count, unsigned long long gate_min,
                  const unsigned long long* gate_source) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int kK = W::kSlots;              // slots of one lane per chunk
  constexpr int kChunkSlots = 32 * kK;       // slots of one warp-wide chunk
  using Cols = ChunkCols<kK>;
  const int nbuf = L.buffers;
  const int cb_pad = L.block_cols + 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);            // [2]
  uint64_t* empty = full + 2;                                         // [2]
  int* next_task = reinterpret_cast<int*>(empty + 2);
  uint64_t* upd = empty + 3;                                          // staged update
  float* sbuf = reinterpret_cast<float*>(smem_raw + kTiledHeader);    // [nbuf][cb_pad]
  int* st = status ? status : &g_tiled_status;
  // A gated launch whose count is below its minimum leaves at once: every CTA
  // reads the same count (written by an earlier launch), so all leave together,
  // before any barrier.
  if (G && *reinterpret_cast<const volatile unsigned long long*>(gate_count) < gate_min)
    return;
  // A gated launch may take its source vector from a pointer an earlier launch left.
  const float* const xin =
      G && gate_source
          ? reinterpret_cast<const float*>(*reinterpret_cast<const volatile unsigned long long*>(gate_source))
          : x0;

  const int c = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int stage_first = L.stage_ptr[c];
  const int stages = L.stage_ptr[c + 1] - stage_first;
  const int task_first = L.task_ptr[c];
  const int task_count = L.task_ptr[c + 1] - task_first;
  const int uses = ticks * stages;  // stage uses of this launch, in order
  // Update rows of this CTA; a staged update needs them in groups of 4 (rows % 4 == 0).
  const int64_t update_lo = L.stage_rows ? 4 * ((L.rows >> 2) * c / gridDim.x) : L.rows * c / gridDim.x;
  const int64_t update_hi =
      L.stage_rows ? 4 * ((L.rows >> 2) * (c + 1) / gridDim.x) : L.rows * (c + 1) / gridDim.x;

  if (threadIdx.x < 4 * nbuf) sbuf[(threadIdx.x >> 2) * cb_pad + L.block_cols + (threadIdx.x & 3)] = 0.0f;
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(full + b, 1);
      mbar_init(empty + b, kConsumerWarps);
    }
    mbar_init(upd, 1);
    *next_task = kConsumerWarps;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  W w = weights;
  if (L.global_scale) w.set_scale(__ldg(L.global_scale));
  const uint64_t pol = evict_first_policy();
  // Bulk L2 prefetch of one task's edges (one lane of the producer warp).  Of
  // a task of several segments only the first segment is prefetched (166k
  // rows x 1.33M columns, 8-chunk tasks of 1-4 chunk segments: 58.4 us per
  // tick with the whole task prefetched, 54.7 us with the first segment).
  auto prefetch_task = [&](const int4& m) {
    const int segment = (m.z >> 26) & 63;
    const int chunks = segment ? segment : m.y;
    if (chunks > 0) {
      prefetch_l2(L.col + m.x, static_cast<uint32_t>(chunks) * kChunkSlots * 2u);
      w.prefetch(m.x, chunks, m.w, ((m.z >> 16) & 0x3FF) * L.split_chunks);
    }
  };
  // Warp w starts every tick with task w; the rest are handed out in order by
  // the shared counter.  The producer warp prefetches tasks into L2 ahead of
  // that counter, and the next tick's first round before the tick ends, so
  // DRAM keeps streaming through the barriers and the update.
  int prefetched = 0;  // producer: tasks of the current tick already prefetched
  int upd_uses = 0;    // completed phases of the staged-update mbarrier
  // Consumer bookkeeping of stage uses (running over all ticks of the launch).
  int waited = -1;  // highest use whose full barrier this warp has observed
  int current = 0;  // lowest use this warp has not left yet
  // Uses are observed in order.  A warp leaves use `current` (arrives on its
  // empty barrier) only after it has seen that use's full barrier, so an
  // arrival can never be counted in the phase of an older use.
  auto observe = [&](int g) {
    if (waited < g) {
      if (!mbar_wait(full + (g % nbuf), (g / nbuf) & 1)) atomicExch(st, 3);
      waited = g;
    }
  };
  auto leave_until = [&](int g) {
    while (current < g) {
      observe(current);
      if (lane == 0 && current < uses - nbuf) mbar_arrive(empty + (current % nbuf));
      ++current;
    }
  };

  for (int tick = 0; tick < ticks; ++tick) {
    const bool exchange = X && px.world > 0;
    const float* x = exchange ? px.gathered[px.rank][tick & 1] : tick == 0 ? xin : out.s.data;
    const int use0 = tick * stages;
    if (warp == kProducerWarp) {
      // All 32 lanes prefetch tasks (each lane one task's metadata load and
      // bulk L2 prefetches); lane 0 also stages the state blocks.
      auto prefetch_upto = [&](int limit) {
        for (; prefetched < limit; prefetched += 32)
          if (prefetched + lane < limit) prefetch_task(__ldg(L.tasks + task_first + prefetched + lane));
        prefetched = limit;
      };
      if (lane == 0) {
        // From the second tick on, the state block must wait until every CTA
        // has written its rows of the previous tick (and read and cleared its
        // row sums): a grid barrier that only this thread of the CTA takes.
        // The consumer warps meanwhile start loading the tick's edges; they
        // touch the row sums only after the staged block arrives, so they
        // are ordered after the barrier through the block's mbarrier.
        if (tick > 0 && !exchange) grid_arrive_wait(L.barrier, st);
        // The state was written by other CTAs' generic stores before the grid
        // barrier; order those writes before this thread's async-proxy reads.
        asm volatile("fence.proxy.async.global;" ::: "memory");
        for (int s = 0; s < stages; ++s) {
          const int g = use0 + s;
          const int b = g % nbuf;
          if (g >= nbuf && !mbar_wait(empty + b, ((g / nbuf) - 1) & 1)) atomicExch(st, 1);
          fence_proxy_async_smem();
          const int64_t first = static_cast<int64_t>(__ldg(L.stage_block + stage_first + s)) *
                                L.block_cols;
          const int count = static_cast<int>(min(static_cast<int64_t>(L.block_cols), L.cols - first));
          const int bulk = count & ~3;  // 16-byte multiple, rest by plain stores
          float* dst = sbuf + b * cb_pad;
          for (int i = bulk; i < count; ++i) dst[i] = x[first + i];
          mbar_arrive_expect_tx(full + b, static_cast<uint32_t>(bulk) * 4u);
          if (bulk > 0) bulk_copy_to_smem(dst, x + first, static_cast<uint32_t>(bulk) * 4u, full + b);
        }
      }
      __syncwarp();
      if (tick == 0) prefetch_upto(min(task_count, L.prefetch_first));  // first round of tick 0
      // L2 prefetch of this tick's tasks, kPrefetchAhead tasks ahead of the
      // hand-out counter, then of the next tick's first round (one task per
      // consumer warp), which keeps DRAM busy across the barriers and the update.
      // Tasks that consumers already took are prefetched too: the prefetched
      // lines enter L2 at normal priority, unlike the evict-first stream, so
      // part of this tick's edges is still in L2 for the next tick (at 166k /
      // 25M fp32 that saves a third of the DRAM reads).  Once every task has
      // been handed out the backlog is dropped, so this warp never holds the
      // CTA back from the grid barrier (layouts of many short tasks).
      const volatile int* handed = next_task;
      long long polls = 0;
      while (prefetched < task_count) {
        const int taken = __shfl_sync(0xffffffffu, *handed, 0);
        if (taken >= task_count + kConsumerWarps) break;  // every consumer found the list empty
        const int limit = min(task_count, taken + L.prefetch_ahead);
        if (prefetched >= limit) {
          if (++polls > kWaitLimit) {  // consumers stalled: stop prefetching
            if (lane == 0) atomicExch(st, 5);
            break;
          }
          __nanosleep(256);
          continue;
        }
        prefetch_upto(min(limit, prefetched + 32));  // one round, then look again
      }
      prefetched = 0;
      if (tick + 1 < ticks) prefetch_upto(min(task_count, L.prefetch_first));
      // The operands of this CTA's update rows, so the update after the grid
      // barrier reads them from L2 (contiguous interior 16-byte spans only).
      if (update && lane < 9) {
        const float* base = nullptr;
        int64_t stride = 0;
        if (lane < 6) {
          base = t.p.data[lane];
          stride = t.p.stride[lane];
        } else {
          const View v = lane == 6 ? (exchange ? View{px.gathered[px.rank][tick & 1] + px.row_offset, 0, 1, 0.0f}
                                     : tick == 0 ? t.s : View{out.s.data, out.s.sb, out.s.sn, 0.0f})
                       : lane == 7 ? (tick == 0 ? t.d : View{out.d.data, out.d.sb, out.d.sn, 0.0f})
                                   : (tick == 0 ? t.a : View{out.a.data, out.a.sb, out.a.sn, 0.0f});
          base = v.data;
          stride = v.sn;
        }
        const int64_t lo = (update_lo + 3) & ~int64_t{3}, hi = update_hi & ~int64_t{3};
        if (base && stride == 1 && reinterpret_cast<uintptr_t>(base) % 16 == 0 && hi > lo)
          prefetch_l2(base + lo, static_cast<uint32_t>((hi - lo) * 4));
      }
      if (lane == 0) {
        // Do not leave the tick while a copy into this CTA's shared memory may
        // be in flight.
        for (int g = max(use0, use0 + stages - nbuf); g < use0 + stages; ++g)
          if (!mbar_wait(full + (g % nbuf), (g / nbuf) & 1)) atomicExch(st, 2);
      }
    } else {
      // ---- load side: task cursor (the next task is fetched one task ahead) --
      // fp32: a task is one or more segments of S chunks (S = 0: one segment),
      // each 32 rows' pieces, lane i's row being word i of the segment's row
      // group.  A segment's row word is read with the issue of its last chunk,
      // straight into that ring entry, where only the store of the segment's
      // sum waits for it: the hand-out chain (grab, then the task) carries no
      // row words, and short pieces come in long tasks (166k rows x 1.33M
      // columns, ~2 chunks per piece: 71.2 -> 57.6 us per tick).  The narrower
      // formats keep one segment per task with its row word (NVFP4: and the
      // lane's decode phase) read with the task: their kernels have fewer
      // registers to spare (fp16 at 166k / 25M: 30.6 -> 32.9 us segmented).
      constexpr bool kPhased = !W::kF32;
      auto grab = [&]() {
        int q = 0;
        if (lane == 0) q = atomicAdd(next_task, 1);
        return __shfl_sync(0xffffffffu, q, 0);
      };
      int next_q = warp < task_count ? warp : task_count;  // first task: static
      int4 next_meta = make_int4(0, 0, 0, 0);
      uint32_t next_row = kRowMask;
      auto fetch = [&]() {
        if (next_q < task_count) {
          const int64_t task = task_first + next_q;
          next_meta = __ldg(L.tasks + task);
          if (kPhased) next_row = static_cast<uint32_t>(__ldg(L.task_rows + task * 32 + lane));
        }
      };
      fetch();
      int slot = 0;          // next slot of this lane to load
      int entry = 0;         // NVFP4: this lane's column in the task's scale table
      int left = 0;          // chunks of the current task not yet loaded
      int chunk = 0;         // NVFP4: index of the next chunk in the lane's piece
      int phase = 0;         // NVFP4 phase of this lane's piece
      uint32_t row = kRowMask;  // NVFP4: the task's row word
      int seg = 0;           // chunks of one segment
      int seg_left = 0;      // chunks of the current segment not yet loaded
      int group = 0;         // row group of the current segment
      uint32_t tag_base = 0;
      // Issue the loads of the next chunk into one ring entry (tag 0: none left).
      auto issue = [&](typename W::Raw& raw, typename Cols::Raw& cols, uint32_t& tag,
                       uint32_t& tag_row) {
        // On a task switch the next task (already fetched) becomes current and
        // the look-ahead is refilled: a shared-counter grab, then the metadata
        // load, which waits for the grab.  For fp32 the refill comes after
        // this chunk's loads, so those never wait behind the grab (166k / 25M
        // 37.4 -> 36.1 us, 1.33M / 200M 653 -> 629 us per tick); the narrower
        // formats refill first, which keeps the hand-out counter, and with it
        // the producer's prefetch window, ahead (NVFP4 33.7 vs 36.5 us).
        constexpr bool kLoadsFirst = W::kF32;
        bool refill = false;
        while (left == 0) {  // warp-uniform
          if (refill) {  // a task without chunks: take the next one now
            next_q = grab();
            fetch();
          }
          if (next_q >= task_count) {
            tag = 0;
            return;
          }
          slot = next_meta.x + lane * kK;
          left = next_meta.y;
          if (kPhased) {
            chunk = ((next_meta.z >> 16) & 0x3FF) * L.split_chunks;  // chunk index within the piece
            entry = next_meta.w + lane;
            phase = static_cast<int>(next_row >> 28);
            row = next_row & kRowMask;
          } else {
            const int s = (next_meta.z >> 26) & 63;
            seg = s ? s : left;
            seg_left = seg;
            group = next_meta.w;
          }
          tag_base = kTagValid | (static_cast<uint32_t>(next_meta.z & 0xFFFF) << kTagStage) |
                     (static_cast<uint32_t>((next_meta.z >> 16) & 0x3FF) << kTagSplit);
          refill = true;
          if (!kLoadsFirst) {
            next_q = grab();
            fetch();
            refill = false;
          }
        }
        const int p = kPhased ? phase + chunk * kK : 0;
        raw = w.load(slot, entry + (p >> 4) * 32, pol);
        cols = Cols::load(L.col, slot, pol);
        if (refill) {
          next_q = grab();
          fetch();
        }
        const bool last = kPhased ? left == 1 : seg_left == 1;
        tag = tag_base | (kPhased ? static_cast<uint32_t>(p & 15) << kTagPhase : 0u) |
              (last ? kTagLast : 0u);
        if (kPhased) {
          tag_row = row;
        } else if (last) {
          tag_row = static_cast<uint32_t>(__ldg(L.task_rows + static_cast<int64_t>(group) * 32 + lane));
          ++group;
          seg_left = seg;
        } else {
          --seg_left;
        }
        slot += kChunkSlots;
        ++chunk;
        --left;
      };

      // ---- the ring ---------------------------------------------------------
      typename W::Raw raw[D];
      typename Cols::Raw cols[D];
      uint32_t tag[D], rows[D];
#pragma unroll
      for (int u = 0; u < D; ++u) issue(raw[u], cols[u], tag[u], rows[u]);
      int stage = -1;
      const float* sb = sbuf;
      float* part = L.part;
      float acc = -0.0f;
      // Entries are issued in order, so once entry 0 is empty all are.
      while (tag[0] & kTagValid) {
#pragma unroll
        for (int u = 0; u < D; ++u) {
          const uint32_t g = tag[u];
          if (g & kTagValid) {
            const int s = static_cast<int>((g >> kTagStage) & 0xFFFFu);
            if (s != stage) {  // warp-uniform
              leave_until(use0 + s);
              observe(use0 + s);
              stage = s;
              sb = sbuf + ((use0 + s) % nbuf) * cb_pad;
              part = L.part + static_cast<int64_t>(__ldg(L.stage_block + stage_first + s)) *
                                  L.splits * L.rows;
            }
            float v[kK];
            w.decode(raw[u], g, v);
#pragma unroll
            for (int e = 0; e < kK; ++e) acc = fmaf(v[e], sb[Cols::at(cols[u], e)], acc);
            if (g & kTagLast) {
              if (rows[u] != kRowMask) part[(g >> kTagSplit) * L.rows + rows[u]] = acc;
              acc = -0.0f;
            }
          }
          issue(raw[u], cols[u], tag[u], rows[u]);
        }
      }
      leave_until(use0 + stages);  // leave every remaining stage of this tick
    }
    __syncthreads();
    if (threadIdx.x == 0) *next_task = kConsumerWarps;
    grid_barrier(L.barrier, st);  // every row sum of this tick is in part

    const int planes = static_cast<int>((L.cols + L.block_cols - 1) / L.block_cols) * L.splits;
    if (L.stage_rows > 0 && update) {
      // Staged update: the state block in shared memory is free until the
      // next tick's staging, so thread 0 bulk-copies the operands of a chunk
      // of this CTA's rows there -- the parameter vectors, s, d, a and every
      // row-sum plane, contiguous runs of 16-byte multiples -- and the threads
      // update the rows from shared memory: one bulk round trip per chunk
      // instead of a round of dependent L2 loads per 1,024 rows.
      const int cap = L.stage_rows;
      float* op = sbuf;  // [6 params | s | d | a | planes][cap]
      for (int64_t c0 = update_lo; c0 < update_hi; c0 += cap) {
        const int rc = static_cast<int>(min(static_cast<int64_t>(cap), update_hi - c0));
        if (threadIdx.x == 0) {
          // Generic writes (the previous tick's d, a and s by this CTA, the
          // row sums by every CTA) before the async-proxy reads; generic
          // reads of shared memory before its async-proxy writes.
          asm volatile("fence.proxy.async.global;" ::: "memory");
          fence_proxy_async_smem();
          const uint32_t bytes = static_cast<uint32_t>(rc) * 4u;
          int copies = 3 + planes;
          for (int i = 0; i < 6; ++i) copies += t.p.stride[i] != 0;
          mbar_arrive_expect_tx(upd, bytes * static_cast<uint32_t>(copies));
          for (int i = 0; i < 6; ++i)  // a parameter broadcast from one value is read directly
            if (t.p.stride[i] != 0) bulk_copy_to_smem(op + i * cap, t.p.data[i] + c0, bytes, upd);
          const float* s_src = exchange ? px.gathered[px.rank][tick & 1] + px.row_offset + c0
                               : tick == 0 ? t.s.data + c0 : out.s.data + c0;
          bulk_copy_to_smem(op + 6 * cap, s_src, bytes, upd);
          bulk_copy_to_smem(op + 7 * cap, (tick == 0 ? t.d.data : out.d.data) + c0, bytes, upd);
          bulk_copy_to_smem(op + 8 * cap, (tick == 0 ? t.a.data : out.a.data) + c0, bytes, upd);
          for (int k = 0; k < planes; ++k)
            bulk_copy_to_smem(op + (9 + k) * cap, L.part + k * L.rows + c0, bytes, upd);
        }
        if (!mbar_wait(upd, upd_uses & 1)) atomicExch(st, 9);
        ++upd_uses;
        auto param = [&](int k, int i) {
          return t.p.stride[k] != 0 ? op[k * cap + i] : __ldg(t.p.data[k]);
        };
        for (int i = threadIdx.x; i < rc; i += blockDim.x) {
          const int64_t n = c0 + i;
          float j = op[9 * cap + i];  // (block, split) order: ((p0 + p1) + p2) + ...
          for (int k = 1; k < planes; ++k) j = j + op[(9 + k) * cap + i];
          for (int k = 0; k < planes; ++k) L.part[n + k * L.rows] = 0.0f;
          const Update q = advance(j, op[6 * cap + i], op[7 * cap + i], op[8 * cap + i],
                                   t.u.at(tick, n), t.v.at(0, n), param(0, i), param(1, i),
                                   param(2, i), param(3, i), param(4, i), param(5, i));
          if (exchange) {
            for (int p = 0; p < px.world; ++p) px.gathered[p][(tick + 1) & 1][px.row_offset + n] = q.s;
          } else {
            out.s.put(0, n, q.s);
          }
          out.d.put(0, n, q.d);
          out.a.put(0, n, q.a);
          if (product.data) product.put(tick, n, q.s);  // a rollout's soma history
        }
        __syncthreads();  // the chunk's operands are read before the next copies
      }
    } else
    // Update of rows [update_lo, update_hi), one row per thread per round:
    // every operand of the row is loaded before any store, so a round costs
    // one memory round trip.  The row sums and the state written by earlier
    // ticks of this launch are read through L2.  (Two rows per round would
    // save a round for the few threads with a second row, but its operands
    // raise the kernel's register need, and the spills that follow slow the
    // streaming loop: 41.0 against 37.6 us per tick at 166k / 25M fp32.)
    for (int64_t n0 = update_lo + threadIdx.x; n0 < update_hi; n0 += blockDim.x) {
      float j[1], s0[1], d0[1], a0[1], u[1], v[1], pr[1][6];
#pragma unroll
      for (int r = 0; r < 1; ++r) {
        const int64_t n = n0 + r * blockDim.x;
        const bool row = n < update_hi;
        s0[r] = d0[r] = a0[r] = u[r] = v[r] = 0.0f;
#pragma unroll
        for (int i = 0; i < 6; ++i) pr[r][i] = 0.0f;
        if (row && update) {  // tick operands exist only for a tick
          if (exchange) {
            s0[r] = __ldcg(px.gathered[px.rank][tick & 1] + px.row_offset + n);
            d0[r] = tick == 0 ? t.d.at(0, n) : __ldcg(out.d.data + n * out.d.sn);
            a0[r] = tick == 0 ? t.a.at(0, n) : __ldcg(out.a.data + n * out.a.sn);
          } else if (tick == 0) {
            s0[r] = t.s.at(0, n);
            d0[r] = t.d.at(0, n);
            a0[r] = t.a.at(0, n);
          } else {
            s0[r] = __ldcg(out.s.data + n * out.s.sn);
            d0[r] = __ldcg(out.d.data + n * out.d.sn);
            a0[r] = __ldcg(out.a.data + n * out.a.sn);
          }
          u[r] = t.u.at(tick, n);  // batch stride = the drive's tick stride (B = 1)
          v[r] = t.v.at(0, n);
#pragma unroll
          for (int i = 0; i < 6; ++i) pr[r][i] = t.p.at(i, n);
        }
        j[r] = 0.0f;
        if (row) {
          const float* p = L.part + n;
          for (int k0 = 0; k0 < planes; k0 += 16) {  // (block, split) order: ((p0 + p1) + p2) + ...
            float sums[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) sums[i] = k0 + i < planes ? __ldcg(p + (k0 + i) * L.rows) : 0.0f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (k0 + i < planes) j[r] = k0 + i == 0 ? sums[i] : j[r] + sums[i];
          }
        }
      }
#pragma unroll
      for (int r = 0; r < 1; ++r) {
        const int64_t n = n0 + r * blockDim.x;
        if (n >= update_hi) continue;
        for (int k = 0; k < planes; ++k) L.part[n + k * L.rows] = 0.0f;
        if (update) {
          const Update q = advance(j[r], s0[r], d0[r], a0[r], u[r], v[r], pr[r][0], pr[r][1],
                                   pr[r][2], pr[r][3], pr[r][4], pr[r][5]);
          if (exchange) {  // the new soma value of row n goes to every rank's next buffer
            for (int p = 0; p < px.world; ++p) px.gathered[p][(tick + 1) & 1][px.row_offset + n] = q.s;
          } else {
            out.s.put(0, n, q.s);
          }
          out.d.put(0, n, q.d);
          out.a.put(0, n, q.a);
          if (product.data) product.put(tick, n, q.s);  // a rollout's soma history
        } else {
          if (G)
            product.data[n * product.sn] += j[r];
          else
            product.put(0, n, j[r]);
        }
      }
    }
    if (exchange) {
      // Every thread's peer stores of this tick precede the CTA barrier; one
      // system-scope fence after it (cumulative over the barrier) orders them
      // all before this CTA's arrival at the ranks' barrier.
      __syncthreads();
      if (warp == kProducerWarp && lane == 0) {
        __threadfence_system();
        peer_barrier(px, L.barrier, tick, st);
      }
    } else {
      __syncthreads();  // this CTA's update is done (the producer's barrier orders it)
    }
  }
}

template <typename W, int D, bool X, bool G>
cudaError_t launch_tiled_kernel(const TiledArgs& L, const W& w, const TickArgs& t,
                                const float* x, const TickOut& out, const Out& product,
                                bool update, int ticks, int* status, int ctas,
                                cudaStream_t stream, const Peers& px,
                                const TiledGate& gate = TiledGate{}) {
  const size_t smem = tiled_smem_bytes(L.block_cols, L.buffers);
  auto kernel = tiled_tick_kernel<W, D, X, G>;
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
  // Cooperative launch: the grid barrier needs every CTA resident at once.
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(ctas);
  config.blockDim = dim3(kTiledThreads);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  attribute[0].id = cudaLaunchAttributeCooperative;
  attribute[0].val.cooperative = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  return cudaLaunchKernelEx(&config, kernel, L, w, t, x, out, product, update, ticks, status, px,
                            gate.count, gate.min, gate.source);
}

template <typename W, int D>
cudaError_t launch_tiled_variant(const TiledArgs& L, const W& w, const TickArgs& t,
                                 const float* x, const TickOut& out, const Out& product,
                                 bool update, int ticks, int* status, int ctas,
                                 cudaStream_t stream, const Peers& px) {
  if (px.world > 0)
    return launch_tiled_kernel<W, D, true, false>(L, w, t, x, out, product, update, ticks, status,
                                                  ctas, stream, px);
  return launch_tiled_kernel<W, D, false, false>(L, w, t, x, out, product, update, ticks, status,
                                                 ctas, stream, px);
}

}  // namespace

size_t tiled_smem_bytes(int block_cols, int buffers) {
  return kTiledHeader + static_cast<size_t>(buffers) * (block_cols + 4) * 4;
}

size_t tiled_workspace_bytes(const nsb_tiled_layout& layout) {
  return 256 + static_cast<size_t>(layout.blocks) * static_cast<size_t>(layout.splits) *
                   static_cast<size_t>(layout.rows) * 4;
}

// The kernel for the layout's weight format at K slots per lane per chunk,
// with a ring of D chunks (K * D = 16 slots of loads in flight per lane).
template <int K, int D>
cudaError_t launch_tiled_format(const nsb_tiled_layout& layout, const TiledArgs& L,
                                const TickArgs& t, const float* x, bool update, int ticks,
                                const TickOut& out, const Out& product, int* status, int ctas,
                                cudaStream_t stream, const Peers& px, const TiledGate& gate) {
  if (gate.count) {  // the hybrid PELS propagate: float32 weights only (checked by the caller)
    return launch_tiled_kernel<ChunkF32<K>, D, false, true>(
        L, ChunkF32<K>{static_cast<const float*>(layout.weight)}, t, x, out, product, update,
        ticks, status, ctas, stream, Peers{}, gate);
  }
  switch (layout.format) {
    case NSB_WEIGHT_F16:
      return launch_tiled_variant<ChunkF16<K>, D>(
          L, ChunkF16<K>{static_cast<const __half*>(layout.weight)}, t, x, out, product, update,
          ticks, status, ctas, stream, px);
    case NSB_WEIGHT_E4M3:
      return launch_tiled_variant<ChunkE4M3<K>, D>(
          L, ChunkE4M3<K>{static_cast<const uint8_t*>(layout.weight), 0.0f}, t, x, out, product,
          update, ticks, status, ctas, stream, px);
    case NSB_WEIGHT_NVFP4:
      return launch_tiled_variant<ChunkNVFP4<K>, D>(
          L, ChunkNVFP4<K>{static_cast<const uint8_t*>(layout.weight), layout.scale_pairs, 0.0f},
          t, x, out, product, update, ticks, status, ctas, stream, px);
    default:
      return launch_tiled_variant<ChunkF32<K>, D>(
          L, ChunkF32<K>{static_cast<const float*>(layout.weight)}, t, x, out, product, update,
          ticks, status, ctas, stream, px);
  }
}

cudaError_t launch_tiled(const nsb_tiled_layout& layout, const TickArgs& t, const float* x,
                         bool update, int ticks, const TickOut& out, const Out& product,
                         void* workspace, int* status, cudaStream_t stream,
                         const nsb_peer_exchange* exchange, const TiledGate& gate) {
  Peers px{};
  if (exchange) {
    px.world = exchange->world;
    px.rank = exchange->rank;
    px.row_offset = exchange->row_offset;
    for (int p = 0; p < exchange->world; ++p) {
      px.gathered[p][0] = exchange->gathered[p][0];
      px.gathered[p][1] = exchange->gathered[p][1];
      px.counters[p] = exchange->counters[p];
    }
    px.epoch = exchange->epoch;
  }
  TiledArgs L;
  L.stage_ptr = layout.stage_ptr;
  L.stage_block = layout.stage_block;
  L.task_ptr = layout.task_ptr;
  L.tasks = reinterpret_cast<const int4*>(layout.tasks);
  L.task_rows = layout.task_rows;
  L.col = layout.col;
  L.global_scale = layout.global_scale;
  L.barrier = static_cast<unsigned long long*>(workspace);
  L.part = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + 256);
  L.block_cols = layout.block_cols;
  L.buffers = layout.buffers;
  L.rows = layout.rows;
  L.cols = layout.cols;
  L.splits = layout.splits;
  L.split_chunks = layout.split_chunks;
  // Prefetch window in tasks: kPrefetchBudget bytes of an average task.
  static const double slot_bytes[4] = {6.0, 4.0, 3.0, 2.5};
  const double task_bytes = layout.n_tasks > 0 ? static_cast<double>(layout.n_slots) *
                                                     slot_bytes[layout.format & 3] / layout.n_tasks
                                               : 1.0;
  const bool prefetch = layout.format != NSB_WEIGHT_F32;
  L.prefetch_ahead = prefetch ? static_cast<int32_t>(
                                    std::min(4096.0, kPrefetchBudget / std::max(task_bytes, 1.0)))
                              : 0;
  L.prefetch_first = prefetch ? kConsumerWarps : 0;
  // Staged update (the tick's row operands bulk-copied into the idle state
  // buffer): every operand a contiguous, 16-byte aligned vector and the rows a
  // multiple of 4 (so each CTA's rows and every plane start on 16 bytes).
  L.stage_rows = 0;
  if (update && !gate.count && layout.rows % 4 == 0) {
    auto ok = [](const void* p, int64_t stride) {
      return p != nullptr && stride == 1 && reinterpret_cast<uintptr_t>(p) % 16 == 0;
    };
    auto ok_param = [&](const float* p, int64_t stride) { return p != nullptr && (stride == 0 || ok(p, stride)); };
    bool staged = ok(t.d.data, t.d.sn) && ok(t.a.data, t.a.sn) && ok(out.d.data, out.d.sn) &&
                  ok(out.a.data, out.a.sn);
    for (int i = 0; i < 6; ++i) staged = staged && ok_param(t.p.data[i], t.p.stride[i]);
    if (exchange) {
      staged = staged && exchange->row_offset % 4 == 0;
      for (int p = 0; p < exchange->world; ++p)
        staged = staged && ok(exchange->gathered[p][0], 1) && ok(exchange->gathered[p][1], 1);
    } else {
      staged = staged && ok(t.s.data, t.s.sn) && (ticks == 1 || ok(out.s.data, out.s.sn));
    }
    const int64_t planes = static_cast<int64_t>(layout.blocks) * layout.splits;
    const int64_t floats = static_cast<int64_t>(layout.buffers) * (layout.block_cols + 4);
    const int64_t cap = floats / (9 + planes) / 4 * 4;
    if (staged && cap >= 64) L.stage_rows = static_cast<int32_t>(std::min<int64_t>(cap, 1 << 20));
  }
  const int ctas = layout.ctas;
  if (layout.chunk == 16) {  // E4M3 / NVFP4 only (checked with the layout)
    switch (layout.format) {
      case NSB_WEIGHT_E4M3:
        return launch_tiled_variant<ChunkE4M3<16>, 2>(
            L, ChunkE4M3<16>{static_cast<const uint8_t*>(layout.weight), 0.0f}, t, x, out,
            product, update, ticks, status, ctas, stream, px);
      default:
        return launch_tiled_variant<ChunkNVFP4<16>, 2>(
            L, ChunkNVFP4<16>{static_cast<const uint8_t*>(layout.weight), layout.scale_pairs, 0.0f},
            t, x, out, product, update, ticks, status, ctas, stream, px);
    }
  }
  return layout.chunk == 8
             ? launch_tiled_format<8, 2>(layout, L, t, x, update, ticks, out, product, status,
                                         ctas, stream, px, gate)
             : launch_tiled_format<4, 4>(layout, L, t, x, update, ticks, out, product, status,
                                         ctas, stream, px, gate);
}

}  // namespace nsb
