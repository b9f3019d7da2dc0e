/*
 * neurosim_b200.h -- C ABI of the B200 dendritic tick library (libneurosim_b200.so).
 *
 * The library replaces the native extension of NeuroSim-GPU for the dendritic
 * hot path.  Its entry points are the FFI a host binds instead of the
 * reference's pybind11 module `neurosim_gpu_native`:
 *
 *   nsb_dendritic_step   <- dendritic_step   (csrc/bindings.cpp:137-142,
 *                                             csrc/compartmental.cu:176-236)
 *   nsb_dendritic_event  <- dendritic_event  (csrc/bindings.cpp:143,
 *                                             csrc/compartmental.cu:238-273)
 *   nsb_csr_propagate    <- the j = W @ x product the runtime needs for its
 *                           persistent current (runtime.py:217-223, which the
 *                           reference computes with cuSPARSE via torch.sparse.mm)
 *
 * Conventions
 *  - Every pointer is a device pointer unless stated otherwise.  Nothing is
 *    retained after a call returns; nothing is allocated by the library.
 *  - A [B,N] operand is an nsb_view: element (b, n) lives at
 *    data[b * batch_stride + n * neuron_stride] (strides in elements, any
 *    sign-free value, 0 for broadcast).  A view whose data is NULL reads as the
 *    constant `scalar` everywhere (the reference's `input=None, input_scalar=x`).
 *  - Outputs are nsb_out views; they must not overlap any input.
 *  - All work is enqueued on `stream` (a cudaStream_t; NULL = legacy default
 *    stream).  No call synchronises the host or allocates, so every call can be
 *    captured into a CUDA graph.
 *  - Return value: NSB_OK, or a negative code after which nothing was
 *    enqueued; nsb_last_error() then returns the message (thread-local).
 *    Invalid arguments are rejected before any launch (the reference raises
 *    RuntimeError from TORCH_CHECK at the same points).
 */
#ifndef NEUROSIM_B200_H
#define NEUROSIM_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define NSB_API __attribute__((visibility("default")))
#else
#define NSB_API
#endif

#define NSB_ABI_VERSION 14

enum nsb_status {
  NSB_OK = 0,
  NSB_ERR_ARGUMENT = -1, /* invalid shape, stride, geometry or null pointer   */
  NSB_ERR_CUDA = -2,     /* a CUDA runtime call failed (message says which)  */
  NSB_ERR_WORKSPACE = -3 /* workspace missing, misaligned or too small        */
};

/* Weight storage of the destination-major CSR (csrc/compartmental.cu:92-119). */
enum nsb_weight_format {
  NSB_WEIGHT_F32 = 0,   /* float[M]                                            */
  NSB_WEIGHT_F16 = 1,   /* IEEE half[M]                                        */
  NSB_WEIGHT_E4M3 = 2,  /* uint8 E4M3FN codes[M] x *global_scale               */
  NSB_WEIGHT_NVFP4 = 3  /* uint8[(M+1)/2]: E2M1 codes, edge 2i in the low
                           nibble of byte i; block_scales[(M+15)/16] E4M3 per
                           16 consecutive edges; x *global_scale               */
};

typedef struct nsb_view {
  const float* data;     /* NULL -> constant `scalar`                          */
  int64_t batch_stride;  /* elements between (b, n) and (b+1, n)              */
  int64_t neuron_stride; /* elements between (b, n) and (b, n+1)              */
  float scalar;
} nsb_view;

typedef struct nsb_out {
  float* data;
  int64_t batch_stride;
  int64_t neuron_stride;
} nsb_out;

/* The six per-neuron parameter vectors, in this order:
 * alpha, gain, dendrite_decay, adaptation_decay, coupling, adaptation_strength
 * (native_compartmental.py:20-23).  stride[i] is in elements. */
typedef struct nsb_params {
  const float* data[6];
  int64_t stride[6];
} nsb_params;

/* Everything one tick reads besides the synaptic current. */
typedef struct nsb_tick {
  int64_t batch;   /* B >= 0                                                    */
  int64_t neurons; /* N >= 1                                                    */
  nsb_view state, dendrite, adaptation; /* s_t, d_t, a_t                        */
  nsb_view input;           /* soma drive u_t (added inside the soma tanh)      */
  nsb_view dendritic_input; /* dendritic drive v_t (added inside the dendrite tanh) */
  nsb_params params;
} nsb_tick;

/* s_{t+1}, d_{t+1}, a_{t+1}. */
typedef struct nsb_tick_out {
  nsb_out state, dendrite, adaptation;
} nsb_tick_out;

/* Destination-major CSR W[dst, src]: the reference's in_rowptr / in_col /
 * in_weight (topology.py:85-93), optionally in a packed weight format. */
typedef struct nsb_csr {
  int64_t n_edges;        /* M                                                 */
  const int32_t* rowptr;  /* [N+1], rowptr[0] = 0, rowptr[N] = M               */
  const int32_t* col;     /* [M] source neuron of each edge                    */
  const void* weight;     /* see nsb_weight_format                             */
  int32_t format;         /* enum nsb_weight_format                            */
  const uint8_t* block_scales; /* NVFP4 only                                   */
  const float* global_scale;   /* E4M3 / NVFP4 only: one float on the device  */
} nsb_csr;

/* Source-major CSR of the same edges for the event scatter: out_rowptr / dst
 * (topology.py:83, 105-115) and a weight per edge.  With weight_index NULL,
 * weight[e] is the weight of source-major edge e (the reference's
 * topology.weight, read coalesced); otherwise weight is the destination-major
 * in_weight and edge e uses weight[weight_index[e]] (the reference call,
 * native_compartmental.py:171-172). */
typedef struct nsb_out_csr {
  int64_t n_edges;
  const int32_t* rowptr;       /* [N+1] */
  const int32_t* dst;          /* [M]   */
  const int32_t* weight_index; /* [M] or NULL */
  const float* weight;         /* [M]   */
} nsb_out_csr;

/* Matrix tick (replaces dendritic_step): j = W @ s_t, then
 *   d' = rd*d + (1-rd)*tanh(j + v)
 *   s' = clamp(alpha*s + (1-alpha)*gain*tanh((1-c)*j + c*d' - k*a + u), 0, 1)
 *   a' = ra*a + (1-ra)*s'
 * `width` is the number of lanes that share one destination row: 4, 8, 16 or 32
 * (the reference accepts 8/16/32; B >= 2 runs 8, 16 or 32, a smaller width
 * meaning 8), or 0 to let the library choose from the mean degree.  The width
 * fixes the order of a row's sum.  One launch; edges are streamed once for
 * every 8 batch rows. */
NSB_API int nsb_dendritic_step(const nsb_tick* tick, const nsb_csr* csr, int32_t width,
                       const nsb_tick_out* out, void* stream);

/* result[b, n] = sum over in-edges of n of w[e] * source[b, col[e]]
 * (one launch, no state update), for any weight format.  Used for the PELS
 * persistent current; with one edge per row and source = 1 it returns the
 * decoded weights themselves. */
NSB_API int nsb_csr_propagate(int64_t batch, int64_t neurons, const nsb_csr* csr,
                      const nsb_view* source, const nsb_out* result, void* stream);

/* Workspace of nsb_dendritic_event, in bytes, for B x N (256-byte aligned,
 * caller-owned device memory; contents need not be initialised). */
NSB_API size_t nsb_dendritic_event_workspace_size(int64_t batch, int64_t neurons);

/* Layout of the workspace head after nsb_dendritic_event has run: */
typedef struct nsb_event_counters {
  uint32_t emitted_sources;   /* (b, n) pairs queued for the scatter            */
  uint32_t reserved;
  uint64_t active_neurons;    /* (b, n) pairs with |s' - emitted| >= theta      */
  uint64_t active_edges;      /* sum of out-degree over active pairs            */
  uint64_t reserved2;
} nsb_event_counters;

/* PELS tick (replaces dendritic_event):
 *   s', d', a' = the matrix-tick update with j = current
 *   active     = |s' - emitted| >= theta[n]
 *   emitted'   = active ? s' : emitted
 *   current   += W @ (active ? s' - emitted : 0)     (in place, float atomics)
 * `current` is a contiguous [B,N] array.  Two launches plus one 32-byte
 * memset; the scatter only visits the out-edges of active sources. */
NSB_API int nsb_dendritic_event(const nsb_tick* tick, float* current, const nsb_view* emitted,
                        const float* theta, int64_t theta_stride,
                        const nsb_out_csr* out_csr, const nsb_tick_out* out,
                        const nsb_out* out_emitted, void* workspace,
                        size_t workspace_bytes, void* stream);

/* Largest B * N that nsb_dendritic_event_noalloc accepts. */
#define NSB_EVENT_NOALLOC_MAX_PAIRS (1 << 20)

/* PELS tick without any device allocation (no counterpart in the reference).
 *
 * Same arguments, checks and results as nsb_dendritic_event, minus the
 * workspace: the counters and the emitter queue live in a fixed array inside
 * the library (256 B + 8 B x NSB_EVENT_NOALLOC_MAX_PAIRS = 8 MiB), which every
 * GPU that loads the library holds until the process exits.  For hosts that
 * cannot hand the library scratch memory: an application whose device memory
 * is all reserved up front by its own pool and that may not allocate during
 * the simulation loop, or a foreign-language host (cgo, JNI, ...) that only
 * holds plain device pointers and has no CUDA allocator of its own.
 *
 * - B * N above NSB_EVENT_NOALLOC_MAX_PAIRS is rejected with NSB_ERR_ARGUMENT.
 * - The first call in each CUDA context (normally once per device, in its
 *   primary context) looks up the array's device address with that device
 *   current (cudaGetSymbolAddress) and keeps it for that context; a call in a
 *   new context (after cudaDeviceReset, or with another driver context
 *   current) looks it up again.  Make the first call before any stream
 *   capture.
 * - All calls on a device share the one array, and each call only clears the
 *   counter head it needs zeroed; calls whose work overlaps on the GPU (other
 *   streams, other threads) race on the array and must be serialised by the
 *   caller.
 * - Calls no cudaMalloc / cudaFree or other allocating routine. */
NSB_API int nsb_dendritic_event_noalloc(const nsb_tick* tick, float* current,
                                        const nsb_view* emitted, const float* theta,
                                        int64_t theta_stride, const nsb_out_csr* out_csr,
                                        const nsb_tick_out* out, const nsb_out* out_emitted,
                                        void* stream);

/* Column-blocked layout of one graph for the B = 1 tick (built by the host,
 * see neurosim_gpu_b200/tiled.py; it re-arranges the destination CSR, the
 * arithmetic is that of nsb_dendritic_step).  It has no counterpart in the
 * reference: it is how this library stores the CSR it is given.
 *  - The gathered columns (`cols` of them) are split into `blocks` blocks of
 *    `block_cols` columns (a multiple of 32, <= 65504).  A stage is one block
 *    and a range of destination rows; CTA c runs stages stage_ptr[c] ..
 *    stage_ptr[c+1]-1 (block stage_block[s]) with `buffers` (1 or 2) state
 *    blocks in shared memory.
 *  - Tasks of CTA c are task_ptr[c] .. task_ptr[c+1]-1.  tasks[4q..4q+3] =
 *    first slot, chunks n, stage (index among the CTA's stages) | h << 16 |
 *    S << 26, and a fourth word.  With `chunk` = C slots per lane per chunk,
 *    a task is split h (h < splits) of 32 rows' pieces in the stage's block:
 *    the lanes' edges C*split_chunks*h + j, j < C*n, lane i's edge
 *    C*split_chunks*h + j at slot first + 32C*(j/C) + C*i + j%C.  With S > 0
 *    (h = 0) the task is n/S such segments of S chunks one after the other,
 *    each for its own 32 rows.
 *    fp32: the fourth word is a row group g, and lane i of segment k owns row
 *    task_rows[32(g+k)+i] & 0x0FFFFFFF (0x0FFFFFFF: no row; S = 0: k = 0).
 *    Other formats (S = 0): lane i owns row task_rows[32q+i] & 0x0FFFFFFF and
 *    the fourth word is the first scale pair (NVFP4).
 *  - col[slot] is the column minus the block start (uint16); padding slots
 *    hold block_cols and weight 0.  n_slots is a multiple of 32C.
 *  - NVFP4: codes are packed two per byte by slot (even slot in the low
 *    nibble).  If lane i's first edge in the block is at CSR position o, its
 *    edge j takes the E4M3 scale of CSR block (o + j) / 16; bits 28..31 of
 *    task_rows[32q+i] hold o % 16, and scale_pairs[first scale pair + 32*b + i]
 *    holds the scales of CSR blocks o/16 + b (low byte) and o/16 + b + 1 (high
 *    byte); past the lane's last edge both are 0.
 *  - Pointer alignment: tasks 16 B; col 2C B; weight 4C B (f32), 2C B (f16),
 *    C B (E4M3), C/2 B (NVFP4).
 *  - The kernels trust the layout's contents (offsets, lengths, rows): pass
 *    layouts made by the builder.  `ctas` must not exceed the SM count: the
 *    tick is a cooperative launch with one CTA per SM. */
typedef struct nsb_tiled_layout {
  int32_t ctas, blocks, block_cols, buffers, format;
  int32_t splits;              /* sub-task splits per block (row-sum planes per block) */
  int32_t split_chunks;        /* chunks of one sub-task                    */
  int32_t chunk;               /* slots of one lane per chunk: 4, 8, or 16 for E4M3 / NVFP4 (C below) */
  int64_t n_stages, n_tasks, n_slots, n_scale_pairs;
  int64_t rows;                /* destination rows                          */
  int64_t cols;                /* length of the gathered source vector      */
  const int32_t* stage_ptr;    /* [ctas+1]            */
  const int32_t* stage_block;  /* [n_stages]          */
  const int32_t* task_ptr;     /* [ctas+1]            */
  const int32_t* tasks;        /* [n_tasks*4]         */
  const int32_t* task_rows;    /* fp32 [row groups*32], else [n_tasks*32] */
  const uint16_t* col;         /* [n_slots]           */
  const void* weight;          /* [n_slots] (NVFP4: [n_slots/2]) */
  const uint16_t* scale_pairs; /* NVFP4: [n_scale_pairs] */
  const float* global_scale;   /* E4M3 / NVFP4        */
} nsb_tiled_layout;

/* Dynamic shared memory one CTA of the tiled tick needs. */
NSB_API size_t nsb_tiled_smem_bytes(int32_t block_cols, int32_t buffers);

/* Device workspace of the tiled calls, in bytes (256-byte aligned, caller-owned):
 * a grid-barrier counter and the row sums of every (block, split) plane.  It must be zero-filled
 * before its first use; every call leaves it zero-filled again, so one
 * workspace serves any number of calls on one stream.  After a call reported
 * a timeout in `status`, zero-fill it again.  Calls that overlap on the GPU
 * need separate workspaces. */
NSB_API size_t nsb_tiled_workspace_size(const nsb_tiled_layout* layout);

/* Matrix tick for B = 1 over a tiled layout (same update as nsb_dendritic_step).
 * `source` is the gathered state vector of layout->cols floats, contiguous and
 * 16-byte aligned; NULL means the tick's own state (then tick->neurons ==
 * layout->cols and the state must be contiguous and aligned).  With a separate
 * source, tick->neurons rows are updated (a rank's rows of a sharded graph).
 * `status` (device int, may be NULL) receives a nonzero code if an internal
 * wait timed out; it is never cleared by the library.  One cooperative launch. */
NSB_API int nsb_dendritic_step_tiled(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                     const float* source, const nsb_tick_out* out,
                                     void* workspace, size_t workspace_bytes, int* status,
                                     void* stream);

/* `ticks` (>= 1) matrix ticks with the same drives in ONE cooperative launch:
 * the first tick reads tick->state / dendrite / adaptation and writes `out`,
 * the later ones update `out` in place.  out->state must be contiguous and
 * 16-byte aligned (it is the gathered source of the later ticks).  Equal to
 * `ticks` calls of nsb_dendritic_step_tiled, bit for bit. */
NSB_API int nsb_dendritic_run_tiled(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                    int64_t ticks, const nsb_tick_out* out, void* workspace,
                                    size_t workspace_bytes, int* status, void* stream);

/* A rollout: `ticks` (>= 1) matrix ticks at B = 1 in ONE cooperative launch,
 * each tick with its own soma drive and its soma state kept (no counterpart in
 * the reference, whose rollouts call the tick once per step: simulate.py:105-107
 * over native_compartmental.py:102-129).  Tick k reads
 * the drive view tick->drive moved on by k * drive_tick_stride floats (0: the
 * same drive every tick; a scalar drive ignores it) and, if `history` is not
 * NULL, writes its new soma state to history[k * history_tick_stride + n]
 * (history_tick_stride >= N).  Otherwise as nsb_dendritic_run_tiled: `out`
 * holds the state after the last tick, which equals `ticks` calls of
 * nsb_dendritic_step_tiled with those drives, bit for bit. */
NSB_API int nsb_dendritic_rollout_tiled(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                        int64_t ticks, int64_t drive_tick_stride,
                                        float* history, int64_t history_tick_stride,
                                        const nsb_tick_out* out, void* workspace,
                                        size_t workspace_bytes, int* status, void* stream);

/* Small graphs: `ticks` (>= 1) matrix ticks at B = 1 on ONE thread-block
 * cluster of 8 CTAs (no counterpart in the reference).  Every CTA keeps the
 * whole state vector and its rows' edges (weights decoded to float32) in
 * shared memory; each tick a CTA updates its rows (each row summed
 * sequentially in CSR order) and writes the new soma values into all 8 CTAs'
 * shared memory (distributed shared memory), then the cluster meets at its
 * hardware barrier.  Nothing goes through global memory between ticks.  The
 * first tick reads the tick's state views, the last writes `out` (any
 * strides).  A CTA stores its rows' edges interleaved by warp, padded to the
 * widest row of each 32 rows: `max_slots` = nsb_cluster_slots(N, host copy of
 * csr->rowptr).  The graph fits when nsb_cluster_smem_bytes(N, max_slots) is
 * at most the device's opt-in shared memory per block (N = 4,096 / M = 65k:
 * about 140 KB).  A `max_slots` below the real value is detected in the
 * kernel, which then writes nothing and sets code 7 in `status` (device int,
 * may be NULL). */
NSB_API int64_t nsb_cluster_slots(int64_t neurons, const int32_t* host_rowptr);
NSB_API size_t nsb_cluster_smem_bytes(int64_t neurons, int64_t max_slots);
NSB_API int nsb_dendritic_run_cluster(const nsb_tick* tick, const nsb_csr* csr, int64_t max_slots,
                                      int64_t ticks, const nsb_tick_out* out, int* status,
                                      void* stream);

/* nsb_dendritic_run_cluster as a rollout (see nsb_dendritic_rollout_tiled; no
 * counterpart in the reference): tick k reads tick->drive moved on by
 * k * drive_tick_stride floats (0: the same drive every tick) and, if
 * `history` is not NULL, writes its new soma state to
 * history[k * history_tick_stride + n] (history_tick_stride >= N). */
NSB_API int nsb_dendritic_rollout_cluster(const nsb_tick* tick, const nsb_csr* csr,
                                          int64_t max_slots, int64_t ticks,
                                          int64_t drive_tick_stride, float* history,
                                          int64_t history_tick_stride, const nsb_tick_out* out,
                                          int* status, void* stream);

/* Up to this many GPUs take part in a peer exchange. */
#define NSB_MAX_PEERS 8

/* The soma exchange of a row-sharded tiled run, done inside the kernel over
 * NVLink instead of an all-gather between launches (no counterpart in the
 * reference, whose runtimes are single-GPU).  Rank r owns global rows
 * [row_offset, row_offset + layout->rows) of a graph whose gathered state has
 * layout->cols floats.  Every rank keeps two gathered buffers; every pointer
 * below is as mapped in THIS process (peers' buffers through CUDA IPC, see
 * nsb_ipc_export / nsb_ipc_import), [rank] being this rank's own. */
typedef struct nsb_peer_exchange {
  int32_t world;               /* ranks, 1..NSB_MAX_PEERS                    */
  int32_t rank;
  int64_t row_offset;
  float* gathered[NSB_MAX_PEERS][2];         /* each rank's two buffers [cols]  */
  unsigned long long* counters[NSB_MAX_PEERS]; /* each rank's arrival counter */
  uint64_t epoch;              /* peer barriers these counters completed before
                                  this call (counter value / world)          */
} nsb_peer_exchange;

/* `ticks` (>= 1) row-sharded matrix ticks in ONE cooperative launch per rank,
 * the soma exchange fused into the kernel: tick t reads the full state from
 * this rank's gathered[rank][t % 2], and the update writes each new s of this
 * rank's rows into gathered[p][(t + 1) % 2] of EVERY rank p (peer stores over
 * NVLink), then waits at a cross-GPU barrier (each rank's counter reaches
 * world * (epoch + t + 1)); after the call every rank's gathered[*][ticks % 2]
 * holds the full new state.  tick->state is ignored (the state comes from the
 * gathered buffer); dendrite / adaptation are read from the tick for the first
 * tick and kept in out->dendrite / out->adaptation (in place) after that;
 * out->state is ignored.  All ranks must make the call with the same ticks,
 * epoch and layout geometry; their kernels wait for each other (bounded: a
 * missing rank ends the call with code 6 in `status`).  The counters must be
 * zero-filled before their first use and the epoch advanced by `ticks` after
 * each call. */
NSB_API int nsb_dendritic_run_tiled_peers(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                          int64_t ticks, const nsb_peer_exchange* exchange,
                                          const nsb_tick_out* out, void* workspace,
                                          size_t workspace_bytes, int* status, void* stream);

/* nsb_dendritic_run_tiled_peers as a rollout (see nsb_dendritic_rollout_tiled):
 * tick k reads this rank's rows' drive tick->drive moved on by
 * k * drive_tick_stride floats and, if `history` is not NULL, writes the new
 * soma state of this rank's rows to history[k * history_tick_stride + row]
 * (history_tick_stride >= layout->rows).  Same exchange, barrier and epoch
 * rules; no counterpart in the reference. */
NSB_API int nsb_dendritic_rollout_tiled_peers(const nsb_tick* tick,
                                              const nsb_tiled_layout* layout, int64_t ticks,
                                              int64_t drive_tick_stride, float* history,
                                              int64_t history_tick_stride,
                                              const nsb_peer_exchange* exchange,
                                              const nsb_tick_out* out, void* workspace,
                                              size_t workspace_bytes, int* status, void* stream);

/* CUDA IPC for the peer exchange: export a device pointer of this process as a
 * 64-byte handle plus the pointer's offset in its allocation, and import such
 * a handle into the current device (peer access enabled) as the allocation's
 * base address.  Release an imported base with nsb_ipc_release. */
NSB_API int nsb_ipc_export(const void* device_ptr, void* handle, uint64_t* offset);
NSB_API int nsb_ipc_import(const void* handle, void** base);
NSB_API int nsb_ipc_release(void* base);

/* Matrix tick of a block of destination rows (any B): the CSR holds those rows
 * (rowptr rebased to 0, col indexing the full source), `source` is the full
 * gathered state [B, n_cols] and the tick's operands are the rows' own.  Used
 * by row-sharded multi-GPU runs; nsb_dendritic_step is the case source = state. */
NSB_API int nsb_dendritic_step_rows(const nsb_tick* tick, const nsb_csr* csr,
                                    const nsb_view* source, int64_t n_cols, int32_t width,
                                    const nsb_tick_out* out, void* stream);

/* result[n] = sum of w[e] * source[col[e]] over the tiled layout (B = 1). */
NSB_API int nsb_tiled_propagate(int64_t neurons, const nsb_tiled_layout* layout,
                                const float* source, float* result, void* workspace,
                                size_t workspace_bytes, int* status, void* stream);

/* Thread-local message of the last failing call ("" if none). */
NSB_API const char* nsb_last_error(void);

/* ---------------------------------------------------------------------------
 * Row-sharded PELS ticks (no counterpart in the reference, which runs on one
 * GPU; each call does what dendritic_event does for one rank's rows).  Rank r
 * owns destination rows [row_offset, row_offset + rows): their s, d, a,
 * emitted state, theta and persistent current.  A tick is two calls:
 *
 * 1. nsb_dendritic_event_rows: the update of the rank's rows with j = current,
 *    the emit rule, and each row's delta (the residual where it emits, else 0)
 *    written to the gathered delta buffer [cols, B] at (row_offset + r) * B + b.
 *    - exchange == NULL: into `delta`; the caller all-gathers the ranks'
 *      slices of it (e.g. ncclAllGather) before step 2.
 *    - exchange != NULL: into every rank's buffer of this tick's parity (peer
 *      stores over NVLink); the kernel's last CTA then adds one to every rank's
 *      arrival counter.  `delta` is not used.
 * 2. nsb_event_scatter_rows: for every nonzero delta of the gathered buffer
 *    (all N sources), current[b, dst - row_offset] += delta * w over the
 *    source's out-edges with a destination in the rank's rows: `csr` is the
 *    source-major out-CSR restricted to them (rowptr [N+1], dst rebased to
 *    [0, rows)).  With an exchange it first waits, bounded, until all ranks
 *    have signalled this tick (timeout: code 6 in `status`, and it goes on).
 *
 * `workspace` (NSB_EVENT_ROWS_WORKSPACE bytes, 8-byte aligned) is zero-filled
 * once and passed to both calls of every tick of one rank; it counts the
 * rank's ticks, so peer-mode calls can be captured into a CUDA graph and
 * replayed.  All ranks' counters start at zero and every rank runs the same
 * ticks.  The float atomics make the summation order of the current
 * nondeterministic (as on one GPU).
 * ------------------------------------------------------------------------- */
#define NSB_EVENT_ROWS_WORKSPACE 256

typedef struct nsb_event_rows {
  int64_t row_offset;      /* global index of the rank's first row            */
  int64_t cols;            /* neuron rows of the gathered delta buffers (>= N) */
  const float* current;    /* [B, rows] contiguous: the rank's rows            */
  nsb_view emitted;        /* [B, rows]                                        */
  const float* theta;      /* the rank's rows of theta                         */
  int64_t theta_stride;
} nsb_event_rows;

typedef struct nsb_delta_exchange {
  int32_t world;                               /* ranks, 1..NSB_MAX_PEERS       */
  int32_t rank;
  float* delta[NSB_MAX_PEERS][2];              /* each rank's two [cols, B] buffers */
  unsigned long long* counters[NSB_MAX_PEERS]; /* each rank's arrival counter    */
} nsb_delta_exchange;

typedef struct nsb_scatter_rows {
  int64_t n_edges;         /* edges with a destination in the rank's rows     */
  const int32_t* rowptr;   /* [N+1] per source                                */
  const int32_t* dst;      /* [n_edges] destination - row_offset              */
  const float* weight;     /* [n_edges]                                       */
} nsb_scatter_rows;

NSB_API int nsb_dendritic_event_rows(const nsb_tick* tick, const nsb_event_rows* ev,
                                     float* delta, const nsb_delta_exchange* exchange,
                                     const nsb_tick_out* out, const nsb_out* out_emitted,
                                     void* workspace, void* stream);
NSB_API int nsb_event_scatter_rows(int64_t batch, int64_t neurons, int64_t rows,
                                   const float* delta, const nsb_scatter_rows* csr,
                                   float* current, const nsb_delta_exchange* exchange,
                                   void* workspace, int* status, void* stream);

/* Hybrid row-sharded PELS tick (B = 1, peer exchange; no counterpart in the
 * reference): the row-sharded tick above with the propagation of the emitted
 * deltas chosen on the device from the tick's activity over ALL ranks, as
 * nsb_dendritic_event_hybrid does on one GPU.  Three calls per tick, on one
 * stream, with the same row-event workspace:
 * 1. nsb_dendritic_event_rows_gated: nsb_dendritic_event_rows with an
 *    exchange, which also sums `out_degree[r]` (the whole graph's out-degree
 *    of the rank's row r) over the rows that emit and adds the rank's sum into
 *    every rank's count of this tick (words 2 + parity of each rank's counter
 *    array: the arrival counter is word 0 of a zero-filled array of at least 4
 *    u64) before it signals its arrival.
 * 2. nsb_event_scatter_rows_gated: after its wait, the scatter returns at once
 *    when the ranks' emitting sources have >= gate_edges (>= 1) out-edges;
 *    else it scatters as nsb_event_scatter_rows does.  It leaves the count and
 *    the address of the tick's gathered delta buffer in the workspace.
 * 3. nsb_tiled_propagate_rows_gated: below the gate it returns at once; at or
 *    above it, current[rows] += W[rows, :] @ delta by the tiled kernel
 *    (`layout`: the float32 tiled layout of the rank's rows x all N columns,
 *    with its workspace; no atomics).
 * All three are always enqueued, so a tick can be captured into a CUDA graph.
 * Every rank must use the same gate_edges. */
NSB_API int nsb_dendritic_event_rows_gated(const nsb_tick* tick, const nsb_event_rows* ev,
                                           const nsb_delta_exchange* exchange,
                                           const int32_t* out_degree, const nsb_tick_out* out,
                                           const nsb_out* out_emitted, void* workspace,
                                           void* stream);
NSB_API int nsb_event_scatter_rows_gated(int64_t neurons, int64_t rows,
                                         const nsb_scatter_rows* csr, float* current,
                                         const nsb_delta_exchange* exchange, uint64_t gate_edges,
                                         void* workspace, int* status, void* stream);
NSB_API int nsb_tiled_propagate_rows_gated(const nsb_tiled_layout* layout, void* tiled_workspace,
                                           size_t tiled_workspace_bytes, float* current,
                                           uint64_t gate_edges, void* workspace, int* status,
                                           void* stream);

/* Weight encoder (replaces encode_sparse_weights, src/neurosim_gpu/precision.py:76-90,
 * for weights in device memory; bit-exact to it).  `format` is NSB_WEIGHT_E4M3
 * (codes: n bytes) or NSB_WEIGHT_NVFP4 (codes: (n+1)/2 bytes, the even-indexed
 * weight in the low nibble; block_scales: (n+15)/16 E4M3 bytes); `global_scale`
 * receives the one float32 scale.  fp8: scale = max(amax/448, FLT_MIN),
 * code = e4m3(clamp(w/scale, +-448)).  NVFP4: g = max(amax/2688, FLT_MIN), per
 * 16 weights bs = e4m3(min(block_amax/(6g), 448)), code = E2M1 of |w|/(g*bs)
 * (ties to the even code) with the sign of w in bit 3.  Weights must be finite.
 * `workspace`: NSB_ENCODE_WORKSPACE bytes of device memory, 4-byte aligned
 * (contents need not be initialised).  Two launches on `stream`. */
#define NSB_ENCODE_WORKSPACE 256
NSB_API int nsb_encode_weights(int32_t format, const float* weight, int64_t n, uint8_t* codes,
                               uint8_t* block_scales, float* global_scale, void* workspace,
                               void* stream);

/* Hybrid PELS tick (B = 1; no counterpart in the reference): the same tick as
 * nsb_dendritic_event, with the propagation of the emitted deltas chosen on the
 * device from this tick's activity.  The advance also writes every neuron's
 * delta (0 where it does not emit) to `dense` ([N] floats, 16-byte aligned).
 * Then, if the emitting sources have fewer than `gate_edges` (>= 1) out-edges
 * in total, the active-edge scatter adds them into `current` (float atomics);
 * otherwise the tiled kernel adds W @ dense into `current` (`layout`: the
 * nsb_tiled_layout of the float32 destination CSR, N x N, with its workspace;
 * deterministic sums).  Both launches are always enqueued and the unselected
 * one returns at once, so the call can be captured into a CUDA graph.
 * `status` receives the tiled kernel's timeout codes (may be NULL). */
NSB_API int nsb_dendritic_event_hybrid(const nsb_tick* tick, float* current,
                                       const nsb_view* emitted, const float* theta,
                                       int64_t theta_stride, const nsb_out_csr* out_csr,
                                       const nsb_tiled_layout* layout, void* tiled_workspace,
                                       size_t tiled_workspace_bytes, float* dense,
                                       uint64_t gate_edges, const nsb_tick_out* out,
                                       const nsb_out* out_emitted, void* workspace,
                                       size_t workspace_bytes, int* status, void* stream);

/* NSB_ABI_VERSION of the loaded library. */
NSB_API int nsb_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* NEUROSIM_B200_H */
