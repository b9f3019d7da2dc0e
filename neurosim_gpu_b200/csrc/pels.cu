// pels.cu -- the PELS tick: advance + emit, then scatter of the emitted deltas.
//
// Launch 1 (event_advance_kernel): one thread per (b, n).  Runs the pointwise
//   update with j = persistent current, applies the emit rule
//   (|s' - emitted| >= theta[n]; csrc/compartmental.cu:142-158) and appends
//   every emitting source with a nonzero delta and out-degree > 0 to a queue
//   (warp-aggregated atomics: one global atomic per warp).  The same pass
//   counts active pairs and their out-edges for the runtime's statistics.
// Launch 2 (event_scatter_kernel): persistent grid; a group of G lanes takes
//   one queued source and adds delta * w to current[b, dst] for each of its
//   out-edges (red.global.add.f32), reading dst and the source-major weight
//   as coalesced 4-edge chunks.  Only active edges are touched, unlike the
//   reference scatter, which starts a warp for every (b, n) pair
//   (csrc/compartmental.cu:160-173).
// Stream order makes launch 1 read the current before launch 2 updates it.
#include <algorithm>
#include <mutex>

#include "nsb_launch.h"

namespace nsb {
namespace {

constexpr int kThreads = 256;

struct Counters {
  unsigned int queued;
  unsigned int reserved;
  unsigned long long active_neurons;
  unsigned long long active_edges;
  unsigned long long reserved2;
};
static_assert(sizeof(Counters) == sizeof(nsb_event_counters), "counter layout");

__global__ void __launch_bounds__(kThreads)
event_advance_kernel(TickArgs t, EventArgs e, TickOut out, Out out_emitted, uint2* queue,
                     Counters* counters) {
  const int lane = threadIdx.x & 31;
  const int64_t neurons = t.neurons;
  const int64_t count = t.batch * neurons;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // Warp-uniform trip count: every lane reaches the ballots below.
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + (threadIdx.x & ~31);
       base < count; base += stride) {
    const int64_t i = base + lane;
    bool enqueue = false;
    bool active = false;
    unsigned int degree = 0;
    float delta = 0.0f;
    if (i < count) {
      const int64_t b = i / neurons;
      const int64_t n = i - b * neurons;
      const Update r = advance_at(t, __ldg(e.current + i), b, n);
      out.s.put(b, n, r.s);
      out.d.put(b, n, r.d);
      out.a.put(b, n, r.a);
      const float previous = e.emitted.at(b, n);
      const float residual = __fsub_rn(r.s, previous);
      active = fabsf(residual) >= __ldg(e.theta + n * e.theta_stride);
      out_emitted.put(b, n, active ? r.s : previous);
      if (e.dense) e.dense[i] = active ? residual : 0.0f;
      if (active) {
        degree = static_cast<unsigned int>(__ldg(e.out_rowptr + n + 1) - __ldg(e.out_rowptr + n));
        delta = residual;
        enqueue = degree > 0 && residual != 0.0f;
      }
    }
    const unsigned int want = __ballot_sync(0xffffffffu, enqueue);
    if (want) {
      const int leader = __ffs(want) - 1;
      unsigned int slot = 0;
      if (lane == leader) slot = atomicAdd(&counters->queued, __popc(want));
      slot = __shfl_sync(0xffffffffu, slot, leader);
      if (enqueue) {
        slot += __popc(want & ((1u << lane) - 1u));
        queue[slot] = make_uint2(static_cast<unsigned int>(i), __float_as_uint(delta));
      }
    }
    const unsigned int act = __ballot_sync(0xffffffffu, active);
    if (act) {
      unsigned long long edges = degree;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) edges += __shfl_xor_sync(0xffffffffu, edges, off);
      if (lane == 0) {
        atomicAdd(&counters->active_neurons, static_cast<unsigned long long>(__popc(act)));
        atomicAdd(&counters->active_edges, edges);
      }
    }
  }
}

__device__ __forceinline__ void red_add(float* p, float v) { atomicAdd(p, v); }

template <int G, bool INDEXED>
__global__ void __launch_bounds__(kThreads)
event_scatter_kernel(EventArgs e, int64_t neurons, const uint2* __restrict__ queue,
                     const Counters* counters, bool vec) {
  const int lg = threadIdx.x % G;
  const int64_t group = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / G;
  const int64_t n_groups = (static_cast<int64_t>(gridDim.x) * blockDim.x) / G;
  // Hybrid tick: at or above the gate the tiled kernel propagates this tick's
  // deltas instead (all threads read the same count, written by the advance).
  if (e.gate_edges &&
      *reinterpret_cast<const volatile unsigned long long*>(&counters->active_edges) >= e.gate_edges)
    return;
  const int64_t queued = *reinterpret_cast<const volatile unsigned int*>(&counters->queued);
  const uint64_t pol = evict_first_policy();
  for (int64_t q = group; q < queued; q += n_groups) {
    const uint2 item = queue[q];
    const int64_t i = item.x;
    const float delta = __uint_as_float(item.y);
    const int64_t b = i / neurons;
    const int64_t n = i - b * neurons;
    float* current = e.current_out + b * neurons;
    const int64_t e0 = __ldg(e.out_rowptr + n);
    const int64_t e1 = __ldg(e.out_rowptr + n + 1);
    if (!INDEXED && vec) {
      const int64_t c_end = (e1 + 3) >> 2;
      for (int64_t c = (e0 >> 2) + lg; c < c_end; c += G) {
        const int64_t first = c << 2;
        int dst[4];
        float w[4];
        if (first + 4 <= e.n_edges) {
          const int4 d4 = stream_load_v4(reinterpret_cast<const int4*>(e.dst) + c, pol);
          const int4 w4 = stream_load_v4(reinterpret_cast<const int4*>(e.weight) + c, pol);
          dst[0] = d4.x; dst[1] = d4.y; dst[2] = d4.z; dst[3] = d4.w;
          w[0] = __int_as_float(w4.x); w[1] = __int_as_float(w4.y);
          w[2] = __int_as_float(w4.z); w[3] = __int_as_float(w4.w);
        } else {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const bool in = first + k < e.n_edges;
            dst[k] = in ? __ldg(e.dst + first + k) : 0;
            w[k] = in ? __ldg(e.weight + first + k) : 0.0f;
          }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (first + k >= e0 && first + k < e1) red_add(current + dst[k], __fmul_rn(delta, w[k]));
      }
    } else {
      for (int64_t edge = e0 + lg; edge < e1; edge += G) {
        const float w = INDEXED ? __ldg(e.weight + __ldg(e.weight_index + edge))
                                : __ldg(e.weight + edge);
        red_add(current + __ldg(e.dst + edge), __fmul_rn(delta, w));
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

template <int G, bool INDEXED>
cudaError_t launch_scatter(const EventArgs& e, int64_t neurons, const uint2* queue,
                           const Counters* counters, bool vec, int sm_count,
                           cudaStream_t stream) {
  auto kernel = event_scatter_kernel<G, INDEXED>;
  static int occupancy = 0;
  if (occupancy == 0) occupancy = resident_blocks(kernel);
  event_scatter_kernel<G, INDEXED><<<sm_count * occupancy, kThreads, 0, stream>>>(
      e, neurons, queue, counters, vec);
  return cudaGetLastError();
}

}  // namespace

size_t event_workspace_bytes(int64_t batch, int64_t neurons) {
  return 256 + static_cast<size_t>(batch * neurons) * sizeof(uint2);
}

// ---------------------------------------------------------------------------
// Scratch for nsb_dendritic_event_noalloc: a fixed array in the library's own
// device image, so that entry point needs no allocation from its caller or
// from the library.  It holds the counter head and the emitter queue of
// NSB_EVENT_NOALLOC_MAX_PAIRS (b, n) pairs, lives on every GPU that loads the
// library until the process exits, and is shared by all calls on that GPU.
// ---------------------------------------------------------------------------
static __device__ __align__(256) unsigned char g_event_scratch[256 + NSB_EVENT_NOALLOC_MAX_PAIRS * 8];

namespace {
std::mutex g_scratch_mutex;

// The scratch address belongs to one CUDA context: after cudaDeviceReset, or
// with a different (non-primary) driver context current, the array has another
// address.  Cached addresses are therefore keyed by the context's unique id
// (cuCtxGetId: never reused within a process), reached through the runtime's
// driver entry point so the library does not link libcuda.
using CtxGetCurrent = int (*)(void**);
using CtxGetId = int (*)(void*, unsigned long long*);
struct ScratchEntry {
  unsigned long long context_id;
  void* address;
};
ScratchEntry g_scratch_address[64] = {};

cudaError_t current_context_id(unsigned long long* id) {
  static CtxGetCurrent get_current = nullptr;
  static CtxGetId get_id = nullptr;
  if (!get_current || !get_id) {
    void* fn_current = nullptr;
    void* fn_id = nullptr;
    cudaDriverEntryPointQueryResult found_current, found_id;
    cudaError_t err = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn_current, cudaEnableDefault,
                                              &found_current);
    if (err != cudaSuccess) return err;
    err = cudaGetDriverEntryPoint("cuCtxGetId", &fn_id, cudaEnableDefault, &found_id);
    if (err != cudaSuccess) return err;
    if (found_current != cudaDriverEntryPointSuccess || found_id != cudaDriverEntryPointSuccess ||
        !fn_current || !fn_id)
      return cudaErrorNotSupported;
    get_current = reinterpret_cast<CtxGetCurrent>(fn_current);
    get_id = reinterpret_cast<CtxGetId>(fn_id);
  }
  void* context = nullptr;
  if (get_current(&context) != 0 || !context) return cudaErrorDeviceUninitialized;
  return get_id(context, id) == 0 ? cudaSuccess : cudaErrorDeviceUninitialized;
}
}  // namespace

// Device address of g_event_scratch in the current context.  The host-side name
// of the array is only a stand-in; the first call in each context asks the
// runtime for the real address (with that context's device current) and keeps
// it for later calls in the same context.
cudaError_t event_noalloc_scratch(void** address) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  unsigned long long context_id = 0;
  err = current_context_id(&context_id);
  if (err == cudaErrorDeviceUninitialized) {
    // No context is current yet: the runtime's symbol lookup makes the
    // device's primary context current, then ask again.
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_event_scratch);
    if (err != cudaSuccess) return err;
    err = current_context_id(&context_id);
  }
  if (err != cudaSuccess) return err;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  ScratchEntry& entry = g_scratch_address[device];
  if (!entry.address || entry.context_id != context_id) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_event_scratch);
    if (err != cudaSuccess) return err;
    entry.address = ptr;
    entry.context_id = context_id;
  }
  *address = entry.address;
  return cudaSuccess;
}

cudaError_t launch_event(const TickArgs& t, const EventArgs& e, const TickOut& out,
                         const Out& out_emitted, void* workspace, cudaStream_t stream) {
  const int64_t count = t.batch * t.neurons;
  if (count == 0) return cudaSuccess;
  DeviceInfo info;
  cudaError_t err = device_info(&info);
  if (err != cudaSuccess) return err;
  auto* counters = static_cast<Counters*>(workspace);
  auto* queue = reinterpret_cast<uint2*>(static_cast<char*>(workspace) + 256);
  err = cudaMemsetAsync(counters, 0, sizeof(Counters), stream);
  if (err != cudaSuccess) return err;

  static int advance_occupancy = 0;
  if (advance_occupancy == 0) advance_occupancy = resident_blocks(event_advance_kernel);
  const int64_t needed = (count + kThreads - 1) / kThreads;
  const int64_t blocks = std::max<int64_t>(
      1, std::min<int64_t>(needed, static_cast<int64_t>(info.sm_count) * advance_occupancy));
  event_advance_kernel<<<static_cast<unsigned>(blocks), kThreads, 0, stream>>>(
      t, e, out, out_emitted, queue, counters);
  err = cudaGetLastError();
  if (err != cudaSuccess) return err;

  const bool indexed = e.weight_index != nullptr;
  const bool vec = !indexed && (reinterpret_cast<uintptr_t>(e.dst) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(e.weight) % 16 == 0);
  const int width = choose_group_width(e.n_edges, t.neurons);
  if (indexed) return launch_scatter<32, true>(e, t.neurons, queue, counters, false, info.sm_count, stream);
  switch (width) {
    case 4: return launch_scatter<4, false>(e, t.neurons, queue, counters, vec, info.sm_count, stream);
    case 8: return launch_scatter<8, false>(e, t.neurons, queue, counters, vec, info.sm_count, stream);
    case 16: return launch_scatter<16, false>(e, t.neurons, queue, counters, vec, info.sm_count, stream);
    default: return launch_scatter<32, false>(e, t.neurons, queue, counters, vec, info.sm_count, stream);
  }
}

}  // namespace nsb
