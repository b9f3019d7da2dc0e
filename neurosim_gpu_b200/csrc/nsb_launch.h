// nsb_launch.h -- host-side launchers shared by the C ABI (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "nsb_device.cuh"

namespace nsb {

// Destination-major CSR as the kernels see it.
struct Csr {
  int64_t n_edges;
  const int32_t* rowptr;
  const int32_t* col;
  const void* weight;
  int32_t format;
  const uint8_t* block_scales;
  const float* global_scale;
};

// Per-device facts, queried once per device.
struct DeviceInfo {
  int sm_count;
};
cudaError_t device_info(DeviceInfo* info);

// Lanes that share one row, chosen from the mean degree (width == 0) or given.
int choose_group_width(int64_t n_edges, int64_t neurons);

// Matrix tick (update = true) or plain product j = W @ x (update = false,
// written to `product`).  `x` is the gathered operand (the state for a tick).
cudaError_t launch_csr(const TickArgs& t, const View& x, const Csr& csr, int width,
                       bool update, const TickOut& out, const Out& product,
                       cudaStream_t stream);

struct EventArgs {
  const float* current;  // contiguous [B,N]; updated in place by the scatter
  float* current_out;
  View emitted;
  const float* theta;
  int64_t theta_stride;
  const int32_t* out_rowptr;
  const int32_t* dst;
  const int32_t* weight_index;  // nullptr: weight is source-major
  const float* weight;
  int64_t n_edges;
  float* dense;                  // hybrid: [B,N] contiguous delta of every pair (0: none), or null
  unsigned long long gate_edges;  // hybrid: the scatter runs only below this many active edges (0: always)
};

// Tiled B = 1 tick with the gathered state staged in shared memory (tiled.cu):
// `ticks` ticks in one cooperative launch (the first reads `t`, later ones run
// in place on `out`).
size_t tiled_smem_bytes(int block_cols, int buffers);
size_t tiled_workspace_bytes(const nsb_tiled_layout& layout);
// Gate of a propagate-only launch (the hybrid PELS tick): the kernel returns at
// once unless *count >= min, and with `accumulate` adds W @ x into `product`.
// With `source`, the launch reads its x pointer from device memory at *source
// (written by an earlier launch on the stream) instead of the argument.
struct TiledGate {
  const unsigned long long* count = nullptr;
  unsigned long long min = 0;
  bool accumulate = false;
  const unsigned long long* source = nullptr;
};

cudaError_t launch_tiled(const nsb_tiled_layout& layout, const TickArgs& t, const float* x,
                         bool update, int ticks, const TickOut& out, const Out& product,
                         void* workspace, int* status, cudaStream_t stream,
                         const nsb_peer_exchange* exchange = nullptr,
                         const TiledGate& gate = TiledGate{});

// Small-graph tick on one thread-block cluster (cluster.cu): `ticks` ticks of
// B = 1 with the state and the edges in the cluster's shared memory.  With a
// nonzero drive_tick_stride tick k reads the drive that many floats on per
// tick; with a history, tick k's new s goes to history.put(k, n).
int64_t cluster_slots(int64_t neurons, const int32_t* host_rowptr);
size_t cluster_smem_bytes(int64_t neurons, int64_t max_slots);
cudaError_t launch_cluster(const TickArgs& t, const Csr& csr, int64_t max_slots, int ticks,
                           const TickOut& out, int* status, cudaStream_t stream,
                           int64_t drive_tick_stride = 0, const Out& history = Out{nullptr, 0, 0});

// Row-sharded PELS (pels_rows.cu).  One rank's rows of the event tick.
struct EventRowsArgs {
  int64_t row_offset;    // global index of the rank's first row
  const float* current;  // [B, rows] contiguous
  View emitted;          // [B, rows]
  const float* theta;    // the rank's rows
  int64_t theta_stride;
  float* delta;          // local mode: the gathered delta buffer [cols, B]
  const int32_t* out_degree = nullptr;  // peer mode: the rows' out-degrees (gated ticks), or null
};

// Every rank's two gathered delta buffers and arrival counters (peer mode).
struct DeltaPeers {
  int32_t world, rank;
  float* delta[NSB_MAX_PEERS][2];
  unsigned long long* counters[NSB_MAX_PEERS];
};

// Head of the caller's row-event workspace (zero-filled once).
struct EventRowsState {
  unsigned long long ticks;  // peer-mode ticks this rank has signalled
  unsigned int done;         // CTAs of the current advance launch that finished
  unsigned int reserved;
  unsigned long long count;         // gated ticks: this launch's emitting out-edges so far
  unsigned long long gate_count;    // gated ticks: all ranks' emitting out-edges of the tick
  unsigned long long gate_source;   // gated ticks: address of the tick's gathered deltas
};

// The source-major out-CSR restricted to the rank's destination rows.
struct ScatterRowsArgs {
  const int32_t* rowptr;  // [N+1]
  const int32_t* dst;     // [M_local], rebased to the rank's rows
  const float* weight;    // [M_local]
  int64_t n_edges;        // M_local
};

cudaError_t launch_event_rows(const TickArgs& t, const EventRowsArgs& e, const TickOut& out,
                              const Out& out_emitted, const DeltaPeers* px,
                              EventRowsState* state, cudaStream_t stream);
// With gate_edges > 0 (peer mode), the scatter returns after its wait when all
// ranks' emitting sources have >= gate_edges out-edges, and CTA 0 leaves that
// count and the tick's delta buffer in `state` for a gated tiled propagate.
cudaError_t launch_event_scatter_rows(int64_t batch, int64_t neurons, int64_t rows,
                                      const float* delta, const ScatterRowsArgs& c,
                                      float* current, const DeltaPeers* px,
                                      EventRowsState* state, int* status,
                                      cudaStream_t stream, unsigned long long gate_edges = 0);

// fp8 / NVFP4 weight encoders (encode.cu); workspace: 4 bytes (the amax word).
cudaError_t launch_encode(int format, const float* weight, int64_t n, uint8_t* codes,
                          uint8_t* block_scales, float* global_scale, void* workspace,
                          cudaStream_t stream);

cudaError_t launch_event(const TickArgs& t, const EventArgs& e, const TickOut& out,
                         const Out& out_emitted, void* workspace, cudaStream_t stream);

// Address of the fixed scratch array used by nsb_dendritic_event_noalloc on the
// current device (pels.cu; first call per device looks it up).
cudaError_t event_noalloc_scratch(void** address);

}  // namespace nsb
