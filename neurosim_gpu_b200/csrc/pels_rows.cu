// pels_rows.cu -- the PELS tick of one rank's rows (row-sharded event ticks).
//
// A rank owns destination rows [row_offset, row_offset + rows) and, for them,
// the soma / dendrite / adaptation / emitted state, theta and the persistent
// current.  One tick is two launches:
//
// 1. event_rows_kernel: thread per (b, r).  The pointwise update with
//    j = current[b, r], the emit rule (|s' - emitted| >= theta; the rule of
//    csrc/compartmental.cu:142-158) and the row's delta (the residual if it
//    emits, else 0), written into the gathered delta buffer at
//    [(row_offset + r) * B + b].  Every row is written every tick, so the
//    gathered buffer needs no clearing.
//    * Local mode: the caller all-gathers the buffers (NCCL) before step 2.
//    * Peer mode (the exchange fused into the kernels): each delta is stored
//      into every rank's buffer of this tick's parity over NVLink; after a CTA
//      barrier one thread per CTA fences at system scope and counts the CTA
//      done, and the last CTA
//      adds one to every rank's arrival counter and advances this rank's tick
//      count (device memory, so CUDA-graph replays need no host epoch).
// 2. event_scatter_rows_kernel: in peer mode every CTA first waits (bounded)
//    until its rank's counter shows all ranks' arrivals for this tick.  Then
//    each warp takes 32 consecutive (source, batch) entries of the gathered
//    delta, ballots the nonzero ones and scatters each one's out-edges with a
//    destination in this rank's range (a source-major CSR filtered to the
//    rank's rows, destinations rebased) into current[b, dst] with float
//    atomics, with G = 8 / 16 / 32 lanes per emitting source (from the mean
//    degree into the rank's rows), 32 / G sources at a time.
//
// The double-buffered delta buffers are safe to reuse: a rank writes parity p
// again two ticks later, only after every rank has passed its wait of the tick
// in between, which follows that rank's scatter of parity p.
#include <algorithm>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kRowThreads = 256;
constexpr long long kDeltaWaitLimit = 1ll << 24;

__device__ __forceinline__ unsigned long long load_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

template <bool X>
__global__ void __launch_bounds__(kRowThreads)
event_rows_kernel(TickArgs t, EventRowsArgs e, TickOut out, Out out_emitted, DeltaPeers px,
                  EventRowsState* state) {
  const int64_t rows = t.neurons;
  const int64_t batch = t.batch;
  const int64_t count = batch * rows;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int parity = 0;
  if (X) parity = static_cast<int>(*reinterpret_cast<volatile unsigned long long*>(&state->ticks) & 1);
  unsigned long long emitting = 0;  // gated ticks: out-edges of this thread's emitting rows
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += stride) {
    const int64_t b = i / rows;
    const int64_t r = i - b * rows;
    const Update q = advance_at(t, __ldg(e.current + b * rows + r), b, r);
    out.s.put(b, r, q.s);
    out.d.put(b, r, q.d);
    out.a.put(b, r, q.a);
    const float previous = e.emitted.at(b, r);
    const float residual = __fsub_rn(q.s, previous);
    const bool active = fabsf(residual) >= __ldg(e.theta + r * e.theta_stride);
    out_emitted.put(b, r, active ? q.s : previous);
    const float delta = active ? residual : 0.0f;
    if (X && e.out_degree && active) emitting += static_cast<unsigned long long>(__ldg(e.out_degree + r));
    const int64_t at = (e.row_offset + r) * batch + b;
    if (X) {
      for (int p = 0; p < px.world; ++p) px.delta[p][parity][at] = delta;
    } else {
      e.delta[at] = delta;
    }
  }
  if (X) {
    // Every thread's peer stores precede the CTA barrier; one system-scope
    // fence after it (cumulative over the barrier) orders them all before the
    // CTA counts itself done.  A fence per thread costs ~ one NVLink round trip
    // each and stalls behind copies in flight.
    if (e.out_degree) {  // one atomic per warp into the launch's count
      for (int o = 16; o > 0; o >>= 1) emitting += __shfl_down_sync(0xffffffffu, emitting, o);
      if ((threadIdx.x & 31) == 0 && emitting) atomicAdd(&state->count, emitting);
    }
    __syncthreads();
    if (threadIdx.x == 0) __threadfence_system();
    if (threadIdx.x == 0 && atomicAdd(&state->done, 1u) == gridDim.x - 1) {
      // The last CTA of this tick: every CTA has counted itself, so the count
      // can start over for the next tick.
      state->done = 0;
      if (e.out_degree) {
        // Every CTA's count preceded its arrival above.  This rank's slot of
        // the next tick's parity starts over (no rank adds to it before this
        // rank's arrival below), and every rank's slot of this tick's parity
        // (words 2 and 3 after its arrival counter) gets this rank's total.
        __threadfence();
        const unsigned long long total = atomicExch(&state->count, 0ull);
        *reinterpret_cast<volatile unsigned long long*>(px.counters[px.rank] + 2 + (parity ^ 1)) = 0ull;
        for (int p = 0; p < px.world; ++p) atomicAdd_system(px.counters[p] + 2 + parity, total);
      }
      __threadfence_system();
      for (int p = 0; p < px.world; ++p) atomicAdd_system(px.counters[p], 1ull);
      atomicAdd(&state->ticks, 1ull);
    }
  }
}

template <bool X, int G>
__global__ void __launch_bounds__(kRowThreads)
event_scatter_rows_kernel(int64_t batch, int64_t neurons, int64_t rows, const float* delta,
                          ScatterRowsArgs c, float* current, DeltaPeers px,
                          EventRowsState* state, int* status, unsigned long long gate_edges) {
  if (X) {
    // Tick k was counted by the advance launch just before this one, so this
    // rank's tick count is k + 1: wait for world * (k + 1) arrivals.
    const unsigned long long ticks = *reinterpret_cast<const volatile unsigned long long*>(&state->ticks);
    delta = px.delta[px.rank][(ticks - 1) & 1];
    if (threadIdx.x == 0) {
      const unsigned long long target = static_cast<unsigned long long>(px.world) * ticks;
      long long polls = 0;
      while (load_acquire_sys(px.counters[px.rank]) < target) {
        if (++polls > (1 << 12)) {
          if (polls > kDeltaWaitLimit) {
            if (status) atomicExch(status, 6);
            break;
          }
          __nanosleep(128);
        }
      }
    }
    __syncthreads();
    if (gate_edges) {
      // All ranks counted this tick's emitting out-edges before they arrived.
      const unsigned long long active = *reinterpret_cast<const volatile unsigned long long*>(
          px.counters[px.rank] + 2 + ((ticks - 1) & 1));
      if (blockIdx.x == 0 && threadIdx.x == 0) {
        state->gate_count = active;
        state->gate_source = reinterpret_cast<unsigned long long>(delta);
      }
      if (active >= gate_edges) return;  // the gated tiled propagate takes this tick
    }
  }
  constexpr int kGroups = 32 / G;  // active sources a warp scatters at once
  const int lane = threadIdx.x & 31;
  const int group = lane / G;
  const int lg = lane % G;
  const int64_t entries = batch * neurons;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  for (int64_t base = warp * 32; base < entries; base += n_warps * 32) {
    const int64_t mine = base + lane;
    // Peer stores land in L2; read the deltas there (not through L1).
    const float d = mine < entries ? __ldcg(delta + mine) : 0.0f;
    unsigned int active = __ballot_sync(0xffffffffu, d != 0.0f);
    while (active) {
      // Group g takes the g-th lowest emitting entry of this round.
      unsigned int rest = active;
      for (int i = 0; i < group && rest; ++i) rest &= rest - 1;
      const int k = rest ? __ffs(rest) - 1 : -1;
      for (int i = 0; i < kGroups && active; ++i) active &= active - 1;
      const float value = __shfl_sync(0xffffffffu, d, k < 0 ? 0 : k);
      if (k < 0) continue;
      const int64_t entry = base + k;
      const int64_t n = entry / batch;
      const int64_t b = entry - n * batch;
      float* row = current + b * rows;
      const int64_t e0 = __ldg(c.rowptr + n);
      const int64_t e1 = __ldg(c.rowptr + n + 1);
      for (int64_t edge = e0 + lg; edge < e1; edge += G)
        atomicAdd(row + __ldg(c.dst + edge), __fmul_rn(value, __ldg(c.weight + edge)));
    }
  }
}

template <typename K>
int resident(K kernel) {
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kRowThreads, 0) != cudaSuccess)
    blocks = 1;
  return std::max(blocks, 1);
}

}  // namespace

cudaError_t launch_event_rows(const TickArgs& t, const EventRowsArgs& e, const TickOut& out,
                              const Out& out_emitted, const DeltaPeers* px,
                              EventRowsState* state, cudaStream_t stream) {
  DeviceInfo info;
  cudaError_t err = device_info(&info);
  if (err != cudaSuccess) return err;
  const int64_t count = t.batch * t.neurons;
  const int64_t needed = std::max<int64_t>(1, (count + kRowThreads - 1) / kRowThreads);
  if (px) {
    static int occupancy = 0;
    if (occupancy == 0) occupancy = resident(event_rows_kernel<true>);
    const int64_t blocks = std::min<int64_t>(needed, int64_t{info.sm_count} * occupancy);
    event_rows_kernel<true><<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(
        t, e, out, out_emitted, *px, state);
  } else {
    static int occupancy = 0;
    if (occupancy == 0) occupancy = resident(event_rows_kernel<false>);
    const int64_t blocks = std::min<int64_t>(needed, int64_t{info.sm_count} * occupancy);
    event_rows_kernel<false><<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(
        t, e, out, out_emitted, DeltaPeers{}, state);
  }
  return cudaGetLastError();
}

namespace {
template <bool X, int G>
cudaError_t scatter_rows_variant(int sm_count, int64_t batch, int64_t neurons, int64_t rows,
                                 const float* delta, const ScatterRowsArgs& c, float* current,
                                 const DeltaPeers& px, EventRowsState* state, int* status,
                                 cudaStream_t stream, unsigned long long gate_edges) {
  static int occupancy = 0;
  if (occupancy == 0) occupancy = resident(event_scatter_rows_kernel<X, G>);
  const int64_t warps = (batch * neurons + 31) / 32;
  const int64_t needed = std::max<int64_t>(1, (warps * 32 + kRowThreads - 1) / kRowThreads);
  const int64_t blocks = std::min<int64_t>(needed, int64_t{sm_count} * occupancy);
  event_scatter_rows_kernel<X, G><<<static_cast<unsigned>(blocks), kRowThreads, 0, stream>>>(
      batch, neurons, rows, delta, c, current, px, state, status, gate_edges);
  return cudaGetLastError();
}

template <bool X>
cudaError_t scatter_rows_width(int sm_count, int64_t n_edges, int64_t batch, int64_t neurons,
                               int64_t rows, const float* delta, const ScatterRowsArgs& c,
                               float* current, const DeltaPeers& px, EventRowsState* state,
                               int* status, cudaStream_t stream, unsigned long long gate_edges) {
  // Lanes per emitting source from the mean out-degree into this rank's rows.
  const double degree = static_cast<double>(n_edges) / static_cast<double>(std::max<int64_t>(neurons, 1));
  if (degree <= 12)
    return scatter_rows_variant<X, 8>(sm_count, batch, neurons, rows, delta, c, current, px, state,
                                      status, stream, gate_edges);
  if (degree <= 24)
    return scatter_rows_variant<X, 16>(sm_count, batch, neurons, rows, delta, c, current, px,
                                       state, status, stream, gate_edges);
  return scatter_rows_variant<X, 32>(sm_count, batch, neurons, rows, delta, c, current, px, state,
                                     status, stream, gate_edges);
}
}  // namespace

cudaError_t launch_event_scatter_rows(int64_t batch, int64_t neurons, int64_t rows,
                                      const float* delta, const ScatterRowsArgs& c,
                                      float* current, const DeltaPeers* px,
                                      EventRowsState* state, int* status,
                                      cudaStream_t stream, unsigned long long gate_edges) {
  DeviceInfo info;
  cudaError_t err = device_info(&info);
  if (err != cudaSuccess) return err;
  if (px)
    return scatter_rows_width<true>(info.sm_count, c.n_edges, batch, neurons, rows, delta, c,
                                    current, *px, state, status, stream, gate_edges);
  return scatter_rows_width<false>(info.sm_count, c.n_edges, batch, neurons, rows, delta, c,
                                   current, DeltaPeers{}, state, status, stream, 0);
}

}  // namespace nsb
