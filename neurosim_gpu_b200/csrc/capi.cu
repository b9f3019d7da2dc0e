// capi.cu -- extern "C" entry points of libneurosim_b200.so (see include/neurosim_b200.h).
//
// Each entry point validates its arguments completely before it enqueues
// anything, mirroring the TORCH_CHECKs of the reference extension
// (csrc/compartmental.cu:29-70, 182-210, 244-256): on failure it returns a
// negative status, leaves the stream untouched and records a message for
// nsb_last_error().
#include <cstdio>
#include <cstring>
#include <string>

#include "nsb_launch.h"

namespace nsb {
size_t event_workspace_bytes(int64_t batch, int64_t neurons);
}  // namespace nsb

namespace {

thread_local std::string g_error;

int fail(int code, const std::string& message) {
  g_error = message;
  return code;
}

int cuda_fail(cudaError_t err, const char* where) {
  return fail(NSB_ERR_CUDA, std::string(where) + ": " + cudaGetErrorName(err) + " (" +
                                cudaGetErrorString(err) + ")");
}

nsb::View to_view(const nsb_view& v) { return {v.data, v.batch_stride, v.neuron_stride, v.scalar}; }
nsb::Out to_out(const nsb_out& o) { return {o.data, o.batch_stride, o.neuron_stride}; }

// Shared checks of the tick operands; fills `t`.
bool check_tick(const nsb_tick* tick, nsb::TickArgs* t) {
  if (!tick) return fail(NSB_ERR_ARGUMENT, "tick arguments are required"), false;
  if (tick->batch < 0 || tick->neurons <= 0)
    return fail(NSB_ERR_ARGUMENT, "state must be [B,N], N > 0"), false;
  if (tick->batch > 0 && (!tick->state.data || !tick->dendrite.data || !tick->adaptation.data))
    return fail(NSB_ERR_ARGUMENT, "state, dendrite and adaptation must be arrays"), false;
  for (int i = 0; i < 6; ++i)
    if (!tick->params.data[i])
      return fail(NSB_ERR_ARGUMENT, "six neuron parameter vectors are required"), false;
  if (tick->batch * tick->neurons >= (int64_t(1) << 32))
    return fail(NSB_ERR_ARGUMENT, "B*N must be below 2^32"), false;
  t->batch = tick->batch;
  t->neurons = tick->neurons;
  t->s = to_view(tick->state);
  t->d = to_view(tick->dendrite);
  t->a = to_view(tick->adaptation);
  t->u = to_view(tick->input);
  t->v = to_view(tick->dendritic_input);
  for (int i = 0; i < 6; ++i) {
    t->p.data[i] = tick->params.data[i];
    t->p.stride[i] = tick->params.stride[i];
  }
  return true;
}

bool check_out(const nsb_out& o, const char* name) {
  if (!o.data) return fail(NSB_ERR_ARGUMENT, std::string(name) + " output is required"), false;
  return true;
}

bool check_csr(const nsb_csr* csr, nsb::Csr* c) {
  if (!csr) return fail(NSB_ERR_ARGUMENT, "CSR arguments are required"), false;
  if (csr->n_edges < 0 || csr->n_edges >= (int64_t(1) << 31))
    return fail(NSB_ERR_ARGUMENT, "invalid CSR geometry: edge count must be in [0, 2^31)"), false;
  if (!csr->rowptr) return fail(NSB_ERR_ARGUMENT, "invalid CSR geometry: rowptr is required"), false;
  if (csr->n_edges > 0 && (!csr->col || !csr->weight))
    return fail(NSB_ERR_ARGUMENT, "invalid CSR geometry: col and weight are required"), false;
  switch (csr->format) {
    case NSB_WEIGHT_F32:
    case NSB_WEIGHT_F16:
      if (csr->block_scales || csr->global_scale)
        return fail(NSB_ERR_ARGUMENT, "invalid floating-point CSR weights: scales given"), false;
      break;
    case NSB_WEIGHT_E4M3:
      if (!csr->global_scale)
        return fail(NSB_ERR_ARGUMENT, "quantized CSR weights require a global scale"), false;
      if (csr->block_scales)
        return fail(NSB_ERR_ARGUMENT, "E4M3 CSR weights take no block scales"), false;
      break;
    case NSB_WEIGHT_NVFP4:
      if (!csr->global_scale)
        return fail(NSB_ERR_ARGUMENT, "quantized CSR weights require a global scale"), false;
      if (csr->n_edges > 0 && !csr->block_scales)
        return fail(NSB_ERR_ARGUMENT, "invalid NVFP4 block scales"), false;
      break;
    default:
      return fail(NSB_ERR_ARGUMENT, "unknown CSR weight format"), false;
  }
  *c = {csr->n_edges, csr->rowptr, csr->col, csr->weight, csr->format, csr->block_scales,
        csr->global_scale};
  return true;
}

bool check_width(int32_t width) {
  if (width == 0 || width == 4 || width == 8 || width == 16 || width == 32) return true;
  fail(NSB_ERR_ARGUMENT, "width must be 4, 8, 16 or 32 (0 = automatic)");
  return false;
}

}  // namespace

extern "C" {

const char* nsb_last_error(void) { return g_error.c_str(); }

int nsb_abi_version(void) { return NSB_ABI_VERSION; }

int nsb_dendritic_step(const nsb_tick* tick, const nsb_csr* csr, int32_t width,
                       const nsb_tick_out* out, void* stream) {
  nsb::TickArgs t;
  nsb::Csr c;
  if (!check_tick(tick, &t) || !check_csr(csr, &c) || !check_width(width)) return NSB_ERR_ARGUMENT;
  if (!out) return fail(NSB_ERR_ARGUMENT, "outputs are required");
  if (t.batch > 0 && (!check_out(out->state, "state") || !check_out(out->dendrite, "dendrite") ||
                      !check_out(out->adaptation, "adaptation")))
    return NSB_ERR_ARGUMENT;
  g_error.clear();
  if (t.batch == 0) return NSB_OK;
  const nsb::TickOut o{to_out(out->state), to_out(out->dendrite), to_out(out->adaptation)};
  const cudaError_t err = nsb::launch_csr(t, t.s, c, width, true, o, nsb::Out{nullptr, 0, 0},
                                          static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_dendritic_step launch");
  return NSB_OK;
}

int nsb_dendritic_step_rows(const nsb_tick* tick, const nsb_csr* csr, const nsb_view* source,
                            int64_t n_cols, int32_t width, const nsb_tick_out* out, void* stream) {
  nsb::TickArgs t;
  nsb::Csr c;
  if (!check_tick(tick, &t) || !check_csr(csr, &c) || !check_width(width)) return NSB_ERR_ARGUMENT;
  if (!source || (t.batch > 0 && !source->data) || n_cols <= 0)
    return fail(NSB_ERR_ARGUMENT, "the gathered source [B, n_cols] is required");
  if (!out) return fail(NSB_ERR_ARGUMENT, "outputs are required");
  if (t.batch > 0 && (!check_out(out->state, "state") || !check_out(out->dendrite, "dendrite") ||
                      !check_out(out->adaptation, "adaptation")))
    return NSB_ERR_ARGUMENT;
  g_error.clear();
  if (t.batch == 0) return NSB_OK;
  const nsb::TickOut o{to_out(out->state), to_out(out->dendrite), to_out(out->adaptation)};
  const cudaError_t err = nsb::launch_csr(t, to_view(*source), c, width, true, o,
                                          nsb::Out{nullptr, 0, 0}, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_dendritic_step_rows launch");
  return NSB_OK;
}

int nsb_csr_propagate(int64_t batch, int64_t neurons, const nsb_csr* csr,
                      const nsb_view* source, const nsb_out* result, void* stream) {
  nsb::Csr c;
  if (batch < 0 || neurons <= 0) return fail(NSB_ERR_ARGUMENT, "source must be [B,N], N > 0");
  if (!check_csr(csr, &c)) return NSB_ERR_ARGUMENT;
  if (!source || !result || (batch > 0 && (!source->data || !result->data)))
    return fail(NSB_ERR_ARGUMENT, "source and result arrays are required");
  g_error.clear();
  if (batch == 0) return NSB_OK;
  nsb::TickArgs t{};
  t.batch = batch;
  t.neurons = neurons;
  const nsb::TickOut none{};
  const cudaError_t err = nsb::launch_csr(t, to_view(*source), c, 0, false, none,
                                          to_out(*result), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_csr_propagate launch");
  return NSB_OK;
}

size_t nsb_tiled_smem_bytes(int32_t block_cols, int32_t buffers) {
  if (block_cols <= 0 || buffers < 1 || buffers > 2) return 0;
  return nsb::tiled_smem_bytes(block_cols, buffers);
}

namespace {

bool aligned(const void* p, uintptr_t bytes) {
  return reinterpret_cast<uintptr_t>(p) % bytes == 0;
}

bool check_tiled(const nsb_tiled_layout* L) {
  if (!L) return fail(NSB_ERR_ARGUMENT, "tiled layout is required"), false;
  if (L->ctas <= 0 || L->blocks <= 0 || L->block_cols <= 0 || L->block_cols % 32 != 0 ||
      L->block_cols > 65504 || (L->buffers != 1 && L->buffers != 2) || L->splits < 1 ||
      L->splits > 1023 || L->split_chunks < 1 || L->n_stages < 0 ||
      L->n_stages >= (int64_t{1} << 24) || L->n_tasks < 0 || L->n_slots < 0 ||
      (L->chunk != 4 && L->chunk != 8 && L->chunk != 16) ||
      (L->chunk == 16 && L->format != NSB_WEIGHT_E4M3 && L->format != NSB_WEIGHT_NVFP4) ||
      L->n_slots % (32 * L->chunk) != 0 ||
      L->n_slots >= (int64_t{1} << 31) || L->rows <= 0 ||
      L->rows >= (int64_t{1} << 28) - 1 || L->cols <= 0 ||
      static_cast<int64_t>(L->blocks) * L->block_cols < L->cols ||
      static_cast<int64_t>(L->blocks - 1) * L->block_cols >= L->cols)
    return fail(NSB_ERR_ARGUMENT, "invalid tiled layout geometry"), false;
  if (!L->stage_ptr || !L->task_ptr || (L->n_stages > 0 && !L->stage_block) ||
      (L->n_tasks > 0 && (!L->tasks || !L->task_rows)) ||
      (L->n_slots > 0 && (!L->col || !L->weight)))
    return fail(NSB_ERR_ARGUMENT, "tiled layout arrays are required"), false;
  static const uintptr_t weight_alignment[4] = {16, 8, 4, 2};  // at chunk 4; x chunk / 4
  if (L->format < 0 || L->format > 3)
    return fail(NSB_ERR_ARGUMENT, "unknown CSR weight format"), false;
  const uintptr_t wide = static_cast<uintptr_t>(L->chunk / 4);
  if (!aligned(L->tasks, 16) || !aligned(L->col, 8 * wide) ||
      !aligned(L->weight, weight_alignment[L->format] * wide))
    return fail(NSB_ERR_ARGUMENT, "tiled layout arrays are misaligned"), false;
  switch (L->format) {
    case NSB_WEIGHT_E4M3:
      if (!L->global_scale) return fail(NSB_ERR_ARGUMENT, "quantized weights require a global scale"), false;
      break;
    case NSB_WEIGHT_NVFP4:
      if (!L->global_scale || (L->n_tasks > 0 && (!L->scale_pairs || L->n_scale_pairs <= 0)) ||
          !aligned(L->scale_pairs, 2))
        return fail(NSB_ERR_ARGUMENT, "invalid NVFP4 tiled layout"), false;
      break;
    default:
      break;
  }
  int device = 0, optin = 0, sms = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err == cudaSuccess)
    err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err != cudaSuccess) return cuda_fail(err, "device attribute query"), false;
  if (nsb::tiled_smem_bytes(L->block_cols, L->buffers) > static_cast<size_t>(optin))
    return fail(NSB_ERR_ARGUMENT, "tiled layout needs more shared memory than a CTA can use"), false;
  if (L->ctas > sms)
    return fail(NSB_ERR_ARGUMENT, "tiled layout has more CTAs than the device has SMs"), false;
  return true;
}

int tiled_status(int code) {
  return g_error.rfind("device attribute query", 0) == 0 ? NSB_ERR_CUDA : code;
}

bool check_workspace(const nsb_tiled_layout* layout, void* workspace, size_t bytes) {
  if (!workspace || !aligned(workspace, 256) || bytes < nsb::tiled_workspace_bytes(*layout))
    return fail(NSB_ERR_WORKSPACE, "tiled workspace missing, misaligned or too small"), false;
  return true;
}

// Checks shared by the tiled tick entry points; fills t and o.
int check_tiled_tick(const nsb_tick* tick, const nsb_tiled_layout* layout, const float** source,
                     const nsb_tick_out* out, void* workspace, size_t workspace_bytes,
                     nsb::TickArgs* t, nsb::TickOut* o) {
  if (!check_tick(tick, t)) return NSB_ERR_ARGUMENT;
  if (t->batch != 1) return fail(NSB_ERR_ARGUMENT, "the tiled tick takes B = 1");
  t->u.sb = 0;  // the kernel reads the drive of tick k at batch index k
  if (!*source) {
    if (t->s.sn != 1)
      return fail(NSB_ERR_ARGUMENT, "the tiled tick needs a contiguous, 16-byte aligned state");
    *source = t->s.data;
  }
  if (!aligned(*source, 16))
    return fail(NSB_ERR_ARGUMENT, "the tiled tick needs a contiguous, 16-byte aligned state");
  if (!out || !check_out(out->state, "state") || !check_out(out->dendrite, "dendrite") ||
      !check_out(out->adaptation, "adaptation"))
    return NSB_ERR_ARGUMENT;
  if (!check_tiled(layout)) return tiled_status(NSB_ERR_ARGUMENT);
  if (layout->rows != t->neurons)
    return fail(NSB_ERR_ARGUMENT, "layout and state neuron counts differ");
  if (!check_workspace(layout, workspace, workspace_bytes)) return NSB_ERR_WORKSPACE;
  *o = nsb::TickOut{to_out(out->state), to_out(out->dendrite), to_out(out->adaptation)};
  return NSB_OK;
}

}  // namespace

size_t nsb_tiled_workspace_size(const nsb_tiled_layout* layout) {
  if (!layout || layout->blocks <= 0 || layout->splits <= 0 || layout->rows <= 0) return 0;
  return nsb::tiled_workspace_bytes(*layout);
}

int nsb_dendritic_step_tiled(const nsb_tick* tick, const nsb_tiled_layout* layout,
                             const float* source, const nsb_tick_out* out, void* workspace,
                             size_t workspace_bytes, int* status, void* stream) {
  nsb::TickArgs t;
  nsb::TickOut o;
  const bool self_source = source == nullptr;
  const int code = check_tiled_tick(tick, layout, &source, out, workspace, workspace_bytes, &t, &o);
  if (code != NSB_OK) return code;
  if (self_source && layout->cols != t.neurons)
    return fail(NSB_ERR_ARGUMENT, "layout and state sizes differ");
  g_error.clear();
  const cudaError_t err = nsb::launch_tiled(*layout, t, source, true, 1, o, nsb::Out{nullptr, 0, 0},
                                            workspace, status, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_dendritic_step_tiled launch");
  return NSB_OK;
}

int nsb_dendritic_run_tiled(const nsb_tick* tick, const nsb_tiled_layout* layout, int64_t ticks,
                            const nsb_tick_out* out, void* workspace, size_t workspace_bytes,
                            int* status, void* stream) {
  if (ticks < 1 || ticks > (int64_t{1} << 24))
    return fail(NSB_ERR_ARGUMENT, "ticks must be in [1, 2^24]");
  nsb::TickArgs t;
  nsb::TickOut o;
  const float* source = nullptr;
  const int code = check_tiled_tick(tick, layout, &source, out, workspace, workspace_bytes, &t, &o);
  if (code != NSB_OK) return code;
  if (layout->cols != t.neurons)
    return fail(NSB_ERR_ARGUMENT, "layout and state sizes differ");
  if (ticks > 1 && (out->state.neuron_stride != 1 || !aligned(out->state.data, 16)))
    return fail(NSB_ERR_ARGUMENT, "multi-tick runs need a contiguous, 16-byte aligned state output");
  g_error.clear();
  const cudaError_t err = nsb::launch_tiled(*layout, t, source, true, static_cast<int>(ticks), o,
                                            nsb::Out{nullptr, 0, 0}, workspace, status,
                                            static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_dendritic_run_tiled launch");
  return NSB_OK;
}

int nsb_dendritic_rollout_tiled(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                int64_t ticks, int64_t drive_tick_stride, float* history,
                                int64_t history_tick_stride, const nsb_tick_out* out,
                                void* workspace, size_t workspace_bytes, int* status,
                                void* stream) {
  if (ticks < 1 || ticks > (int64_t{1} << 24))
    return fail(NSB_ERR_ARGUMENT, "ticks must be in [1, 2^24]");
  if (drive_tick_stride < 0 || drive_tick_stride > (int64_t{1} << 40))
    return fail(NSB_ERR_ARGUMENT, "drive_tick_stride must be in [0, 2^40]");
  nsb::TickArgs t;
  nsb::TickOut o;
  const float* source = nullptr;
  const int code = check_tiled_tick(tick, layout, &source, out, workspace, workspace_bytes, &t, &o);
  if (code != NSB_OK) return code;
  if (layout->cols != t.neurons)
    return fail(NSB_ERR_ARGUMENT, "layout and state sizes differ");
  if (ticks > 1 && (out->state.neuron_stride != 1 || !aligned(out->state.data, 16)))
    return fail(NSB_ERR_ARGUMENT, "multi-tick runs need a contiguous, 16-byte aligned state output");
  if (history && (history_tick_stride < t.neurons || history_tick_stride > (int64_t{1} << 40)))
    return fail(NSB_ERR_ARGUMENT, "history_tick_stride must be in [neurons, 2^40]");
  if (t.u.data) t.u.sb = drive_tick_stride;
  g_error.clear();
  const cudaError_t err = nsb::launch_tiled(*layout, t, source, true, static_cast<int>(ticks), o,
                                            nsb::Out{history, history ? history_tick_stride : 0, 1},
                                            workspace, status, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_dendritic_rollout_tiled launch");
  return NSB_OK;
}

namespace {

// The checks and the launch shared by the two peer-exchange entry points.
int run_tiled_peers(const nsb_tick* tick, const nsb_tiled_layout* layout, int64_t ticks,
                    int64_t drive_tick_stride, float* history, int64_t history_tick_stride,
                    const nsb_peer_exchange* x, const nsb_tick_out* out, void* workspace,
                    size_t workspace_bytes, int* status, void* stream, const char* name) {
  if (ticks < 1 || ticks > (int64_t{1} << 24))
    return fail(NSB_ERR_ARGUMENT, "ticks must be in [1, 2^24]");
  if (drive_tick_stride < 0 || drive_tick_stride > (int64_t{1} << 40))
    return fail(NSB_ERR_ARGUMENT, "drive_tick_stride must be in [0, 2^40]");
  if (!x || x->world < 1 || x->world > NSB_MAX_PEERS || x->rank < 0 || x->rank >= x->world)
    return fail(NSB_ERR_ARGUMENT, "invalid peer exchange: world / rank");
  for (int p = 0; p < x->world; ++p)
    if (!x->gathered[p][0] || !x->gathered[p][1] || !x->counters[p] ||
        !aligned(x->gathered[p][0], 16) || !aligned(x->gathered[p][1], 16) ||
        !aligned(x->counters[p], 8))
      return fail(NSB_ERR_ARGUMENT, "invalid peer exchange: buffers missing or misaligned");
  nsb::TickArgs t;
  nsb::TickOut o;
  const float* source = x->gathered[x->rank][0];
  const int code = check_tiled_tick(tick, layout, &source, out, workspace, workspace_bytes, &t, &o);
  if (code != NSB_OK) return code;
  if (x->row_offset < 0 || x->row_offset + layout->rows > layout->cols)
    return fail(NSB_ERR_ARGUMENT, "invalid peer exchange: rows outside the gathered state");
  if (history && (history_tick_stride < t.neurons || history_tick_stride > (int64_t{1} << 40)))
    return fail(NSB_ERR_ARGUMENT, "history_tick_stride must be in [rows, 2^40]");
  if (t.u.data) t.u.sb = drive_tick_stride;
  g_error.clear();
  const cudaError_t err = nsb::launch_tiled(*layout, t, source, true, static_cast<int>(ticks), o,
                                            nsb::Out{history, history ? history_tick_stride : 0, 1},
                                            workspace, status, static_cast<cudaStream_t>(stream), x);
  if (err != cudaSuccess) return cuda_fail(err, name);
  return NSB_OK;
}

}  // namespace

int nsb_dendritic_run_tiled_peers(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                  int64_t ticks, const nsb_peer_exchange* x,
                                  const nsb_tick_out* out, void* workspace,
                                  size_t workspace_bytes, int* status, void* stream) {
  return run_tiled_peers(tick, layout, ticks, 0, nullptr, 0, x, out, workspace, workspace_bytes,
                         status, stream, "nsb_dendritic_run_tiled_peers launch");
}

int nsb_dendritic_rollout_tiled_peers(const nsb_tick* tick, const nsb_tiled_layout* layout,
                                      int64_t ticks, int64_t drive_tick_stride, float* history,
                                      int64_t history_tick_stride, const nsb_peer_exchange* x,
                                      const nsb_tick_out* out, void* workspace,
                                      size_t workspace_bytes, int* status, void* stream) {
  return run_tiled_peers(tick, layout, ticks, drive_tick_stride, history, history_tick_stride, x,
                         out, workspace, workspace_bytes, status, stream,
                         "nsb_dendritic_rollout_tiled_peers launch");
}

int64_t nsb_cluster_slots(int64_t neurons, const int32_t* host_rowptr) {
  if (neurons <= 0 || neurons >= (int64_t{1} << 31) || !host_rowptr) return -1;
  return nsb::cluster_slots(neurons, host_rowptr);
}

size_t nsb_cluster_smem_bytes(int64_t neurons, int64_t max_slots) {
  if (neurons <= 0 || neurons >= (int64_t{1} << 31) || max_slots < 0 ||
      max_slots >= (int64_t{1} << 31))
    return 0;
  return nsb::cluster_smem_bytes(neurons, max_slots);
}

namespace {

int run_cluster(const nsb_tick* tick, const nsb_csr* csr, int64_t max_slots, int64_t ticks,
                int64_t drive_tick_stride, float* history, int64_t history_tick_stride,
                const nsb_tick_out* out, int* status, void* stream, const char* name) {
  if (ticks < 1 || ticks > (int64_t{1} << 30))
    return fail(NSB_ERR_ARGUMENT, "ticks must be in [1, 2^30]");
  if (drive_tick_stride < 0 || drive_tick_stride > (int64_t{1} << 40))
    return fail(NSB_ERR_ARGUMENT, "drive_tick_stride must be in [0, 2^40]");
  nsb::TickArgs t;
  if (!check_tick(tick, &t)) return NSB_ERR_ARGUMENT;
  if (t.batch != 1) return fail(NSB_ERR_ARGUMENT, "the cluster tick takes B = 1");
  nsb::Csr c;
  if (!check_csr(csr, &c)) return NSB_ERR_ARGUMENT;
  if (!out || !check_out(out->state, "state") || !check_out(out->dendrite, "dendrite") ||
      !check_out(out->adaptation, "adaptation"))
    return NSB_ERR_ARGUMENT;
  if (max_slots < 0 || max_slots >= (int64_t{1} << 31))
    return fail(NSB_ERR_ARGUMENT, "max_slots must be in [0, 2^31)");
  if (history && (history_tick_stride < t.neurons || history_tick_stride > (int64_t{1} << 40)))
    return fail(NSB_ERR_ARGUMENT, "history_tick_stride must be in [neurons, 2^40]");
  int device = 0, optin = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err == cudaSuccess)
    err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
  if (err != cudaSuccess) return cuda_fail(err, "device attribute query");
  if (nsb::cluster_smem_bytes(t.neurons, max_slots) > static_cast<size_t>(optin))
    return fail(NSB_ERR_ARGUMENT, "the graph does not fit the cluster tick's shared memory");
  g_error.clear();
  const nsb::TickOut o{to_out(out->state), to_out(out->dendrite), to_out(out->adaptation)};
  err = nsb::launch_cluster(t, c, max_slots, static_cast<int>(ticks), o, status,
                            static_cast<cudaStream_t>(stream), drive_tick_stride,
                            nsb::Out{history, history ? history_tick_stride : 0, 1});
  if (err != cudaSuccess) return cuda_fail(err, name);
  return NSB_OK;
}

}  // namespace

int nsb_dendritic_run_cluster(const nsb_tick* tick, const nsb_csr* csr, int64_t max_slots,
                              int64_t ticks, const nsb_tick_out* out, int* status,
                              void* stream) {
  return run_cluster(tick, csr, max_slots, ticks, 0, nullptr, 0, out, status, stream,
                     "nsb_dendritic_run_cluster launch");
}

int nsb_dendritic_rollout_cluster(const nsb_tick* tick, const nsb_csr* csr, int64_t max_slots,
                                  int64_t ticks, int64_t drive_tick_stride, float* history,
                                  int64_t history_tick_stride, const nsb_tick_out* out,
                                  int* status, void* stream) {
  return run_cluster(tick, csr, max_slots, ticks, drive_tick_stride, history,
                     history_tick_stride, out, status, stream,
                     "nsb_dendritic_rollout_cluster launch");
}

namespace {
// cuMemGetAddressRange through the runtime's driver entry point (no -lcuda).
using AddressRange = int (*)(unsigned long long*, size_t*, unsigned long long);
}  // namespace

int nsb_ipc_export(const void* device_ptr, void* handle, uint64_t* offset) {
  if (!device_ptr || !handle || !offset) return fail(NSB_ERR_ARGUMENT, "ipc export: null argument");
  static AddressRange range = nullptr;
  if (!range) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult found;
    const cudaError_t err = cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault,
                                                    &found);
    if (err != cudaSuccess || found != cudaDriverEntryPointSuccess || !fn)
      return fail(NSB_ERR_CUDA, "ipc export: cuMemGetAddressRange is unavailable");
    range = reinterpret_cast<AddressRange>(fn);
  }
  unsigned long long base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<unsigned long long>(device_ptr)) != 0)
    return fail(NSB_ERR_ARGUMENT, "ipc export: not a device allocation");
  cudaIpcMemHandle_t h;
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return cuda_fail(err, "ipc export");
  std::memcpy(handle, &h, sizeof(h));
  *offset = reinterpret_cast<unsigned long long>(device_ptr) - base;
  return NSB_OK;
}

int nsb_ipc_import(const void* handle, void** base) {
  if (!handle || !base) return fail(NSB_ERR_ARGUMENT, "ipc import: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t err = cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return cuda_fail(err, "ipc import");
  return NSB_OK;
}

int nsb_ipc_release(void* base) {
  if (!base) return fail(NSB_ERR_ARGUMENT, "ipc release: null base");
  const cudaError_t err = cudaIpcCloseMemHandle(base);
  if (err != cudaSuccess) return cuda_fail(err, "ipc release");
  return NSB_OK;
}

int nsb_tiled_propagate(int64_t neurons, const nsb_tiled_layout* layout, const float* source,
                        float* result, void* workspace, size_t workspace_bytes, int* status,
                        void* stream) {
  if (neurons <= 0) return fail(NSB_ERR_ARGUMENT, "source must be [1,N], N > 0");
  if (!source || !result) return fail(NSB_ERR_ARGUMENT, "source and result arrays are required");
  if (!aligned(source, 16))
    return fail(NSB_ERR_ARGUMENT, "the tiled product needs a 16-byte aligned source");
  if (!check_tiled(layout)) return tiled_status(NSB_ERR_ARGUMENT);
  if (layout->cols != neurons || layout->rows != neurons)
    return fail(NSB_ERR_ARGUMENT, "layout and source sizes differ");
  if (!check_workspace(layout, workspace, workspace_bytes)) return NSB_ERR_WORKSPACE;
  g_error.clear();
  nsb::TickArgs t{};
  t.batch = 1;
  t.neurons = neurons;
  const cudaError_t err = nsb::launch_tiled(*layout, t, source, false, 1, nsb::TickOut{},
                                            nsb::Out{result, 0, 1}, workspace, status,
                                            static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_tiled_propagate launch");
  return NSB_OK;
}

size_t nsb_dendritic_event_workspace_size(int64_t batch, int64_t neurons) {
  if (batch < 0 || neurons < 0) return 0;
  return nsb::event_workspace_bytes(batch, neurons);
}

namespace {
// The PELS tick, with or without the hybrid propagation (hybrid == nullptr:
// the scatter handles every tick).
struct HybridArgs {
  const nsb_tiled_layout* layout;
  void* tiled_workspace;
  size_t tiled_workspace_bytes;
  float* dense;
  uint64_t gate_edges;
  int* status;
};

int event_tick(const nsb_tick* tick, float* current, const nsb_view* emitted, const float* theta,
               int64_t theta_stride, const nsb_out_csr* out_csr, const nsb_tick_out* out,
               const nsb_out* out_emitted, void* workspace, size_t workspace_bytes,
               const HybridArgs* hybrid, void* stream, const char* name) {
  nsb::TickArgs t;
  if (!check_tick(tick, &t)) return NSB_ERR_ARGUMENT;
  if (t.batch > 0 && (!current || !emitted || !emitted->data))
    return fail(NSB_ERR_ARGUMENT, "persistent current and emitted state are required");
  if (!theta) return fail(NSB_ERR_ARGUMENT, "theta must have N values");
  if (!out_csr || !out_csr->rowptr || out_csr->n_edges < 0 || out_csr->n_edges >= (int64_t(1) << 31) ||
      (out_csr->n_edges > 0 && (!out_csr->dst || !out_csr->weight)))
    return fail(NSB_ERR_ARGUMENT, "invalid event topology geometry");
  if (!out || !out_emitted) return fail(NSB_ERR_ARGUMENT, "outputs are required");
  if (t.batch > 0 && (!check_out(out->state, "state") || !check_out(out->dendrite, "dendrite") ||
                      !check_out(out->adaptation, "adaptation") ||
                      !check_out(*out_emitted, "emitted")))
    return NSB_ERR_ARGUMENT;
  const size_t need = nsb::event_workspace_bytes(t.batch, t.neurons);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return fail(NSB_ERR_WORKSPACE, "event workspace must be 256-byte aligned and at least " +
                                       std::to_string(need) + " bytes");
  if (hybrid) {
    if (t.batch != 1) return fail(NSB_ERR_ARGUMENT, "the hybrid PELS tick takes B = 1");
    if (!check_tiled(hybrid->layout)) return tiled_status(NSB_ERR_ARGUMENT);
    if (hybrid->layout->rows != t.neurons || hybrid->layout->cols != t.neurons ||
        hybrid->layout->format != NSB_WEIGHT_F32)
      return fail(NSB_ERR_ARGUMENT, "the hybrid layout must be the N x N float32 destination CSR");
    if (!check_workspace(hybrid->layout, hybrid->tiled_workspace, hybrid->tiled_workspace_bytes))
      return NSB_ERR_WORKSPACE;
    if (!hybrid->dense || !aligned(hybrid->dense, 16))
      return fail(NSB_ERR_ARGUMENT, "the hybrid tick needs a 16-byte aligned [N] delta buffer");
    if (hybrid->gate_edges == 0)
      return fail(NSB_ERR_ARGUMENT, "the hybrid gate must be at least one edge");
  }
  g_error.clear();
  if (t.batch == 0) return NSB_OK;
  nsb::EventArgs e{};
  e.current = current;
  e.current_out = current;
  e.emitted = to_view(*emitted);
  e.theta = theta;
  e.theta_stride = theta_stride;
  e.out_rowptr = out_csr->rowptr;
  e.dst = out_csr->dst;
  e.weight_index = out_csr->weight_index;
  e.weight = out_csr->weight;
  e.n_edges = out_csr->n_edges;
  e.dense = hybrid ? hybrid->dense : nullptr;
  e.gate_edges = hybrid ? hybrid->gate_edges : 0;
  const nsb::TickOut o{to_out(out->state), to_out(out->dendrite), to_out(out->adaptation)};
  cudaError_t err = nsb::launch_event(t, e, o, to_out(*out_emitted), workspace,
                                      static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, name);
  if (hybrid) {
    // Ticks at or above the gate: current += W @ delta by the tiled kernel
    // (the scatter has returned for them; below the gate this launch returns).
    nsb::TiledGate gate;
    gate.count = reinterpret_cast<const unsigned long long*>(
        &static_cast<const nsb_event_counters*>(workspace)->active_edges);
    gate.min = hybrid->gate_edges;
    gate.accumulate = true;
    nsb::TickArgs none{};
    none.batch = 1;
    none.neurons = t.neurons;
    err = nsb::launch_tiled(*hybrid->layout, none, hybrid->dense, false, 1, nsb::TickOut{},
                            nsb::Out{current, 0, 1}, hybrid->tiled_workspace, hybrid->status,
                            static_cast<cudaStream_t>(stream), nullptr, gate);
    if (err != cudaSuccess) return cuda_fail(err, name);
  }
  return NSB_OK;
}
}  // namespace

int nsb_dendritic_event(const nsb_tick* tick, float* current, const nsb_view* emitted,
                        const float* theta, int64_t theta_stride, const nsb_out_csr* out_csr,
                        const nsb_tick_out* out, const nsb_out* out_emitted, void* workspace,
                        size_t workspace_bytes, void* stream) {
  return event_tick(tick, current, emitted, theta, theta_stride, out_csr, out, out_emitted,
                    workspace, workspace_bytes, nullptr, stream, "nsb_dendritic_event launch");
}

int nsb_dendritic_event_hybrid(const nsb_tick* tick, float* current, const nsb_view* emitted,
                               const float* theta, int64_t theta_stride,
                               const nsb_out_csr* out_csr, const nsb_tiled_layout* layout,
                               void* tiled_workspace, size_t tiled_workspace_bytes, float* dense,
                               uint64_t gate_edges, const nsb_tick_out* out,
                               const nsb_out* out_emitted, void* workspace,
                               size_t workspace_bytes, int* status, void* stream) {
  const HybridArgs hybrid{layout, tiled_workspace, tiled_workspace_bytes, dense, gate_edges,
                          status};
  return event_tick(tick, current, emitted, theta, theta_stride, out_csr, out, out_emitted,
                    workspace, workspace_bytes, &hybrid, stream,
                    "nsb_dendritic_event_hybrid launch");
}

namespace {
bool check_delta_exchange(const nsb_delta_exchange* x, nsb::DeltaPeers* px) {
  if (x->world < 1 || x->world > NSB_MAX_PEERS || x->rank < 0 || x->rank >= x->world)
    return fail(NSB_ERR_ARGUMENT, "delta exchange: world must be 1..8 and rank in [0, world)"),
           false;
  px->world = x->world;
  px->rank = x->rank;
  for (int p = 0; p < x->world; ++p) {
    if (!x->delta[p][0] || !x->delta[p][1] || !x->counters[p])
      return fail(NSB_ERR_ARGUMENT, "delta exchange: every rank needs two buffers and a counter"),
             false;
    px->delta[p][0] = x->delta[p][0];
    px->delta[p][1] = x->delta[p][1];
    px->counters[p] = x->counters[p];
  }
  return true;
}

bool check_rows_workspace(void* workspace) {
  if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 8 != 0)
    return fail(NSB_ERR_WORKSPACE, "row-event workspace must be 8-byte aligned"), false;
  return true;
}
}  // namespace

namespace {
int event_rows(const nsb_tick* tick, const nsb_event_rows* ev, float* delta,
               const nsb_delta_exchange* exchange, const int32_t* out_degree,
               const nsb_tick_out* out, const nsb_out* out_emitted, void* workspace,
               void* stream, const char* name) {
  nsb::TickArgs t;
  if (!check_tick(tick, &t)) return NSB_ERR_ARGUMENT;
  if (!ev) return fail(NSB_ERR_ARGUMENT, "row-event arguments are required");
  if (ev->row_offset < 0 || ev->cols < ev->row_offset + t.neurons ||
      ev->cols * t.batch >= (int64_t(1) << 40))
    return fail(NSB_ERR_ARGUMENT, "rows must lie in [0, cols) of the delta buffer");
  if (t.batch > 0 && (!ev->current || !ev->emitted.data))
    return fail(NSB_ERR_ARGUMENT, "persistent current and emitted state are required");
  if (!ev->theta) return fail(NSB_ERR_ARGUMENT, "theta must have a value per row");
  if (!exchange && !delta) return fail(NSB_ERR_ARGUMENT, "a delta buffer or an exchange is required");
  nsb::DeltaPeers px{};
  if (exchange && !check_delta_exchange(exchange, &px)) return NSB_ERR_ARGUMENT;
  if (!out || !out_emitted) return fail(NSB_ERR_ARGUMENT, "outputs are required");
  if (t.batch > 0 && (!check_out(out->state, "state") || !check_out(out->dendrite, "dendrite") ||
                      !check_out(out->adaptation, "adaptation") ||
                      !check_out(*out_emitted, "emitted")))
    return NSB_ERR_ARGUMENT;
  if (!check_rows_workspace(workspace)) return NSB_ERR_WORKSPACE;
  g_error.clear();
  if (t.batch == 0) return NSB_OK;
  nsb::EventRowsArgs e;
  e.row_offset = ev->row_offset;
  e.current = ev->current;
  e.emitted = to_view(ev->emitted);
  e.theta = ev->theta;
  e.theta_stride = ev->theta_stride;
  e.delta = delta;
  e.out_degree = out_degree;
  const nsb::TickOut o{to_out(out->state), to_out(out->dendrite), to_out(out->adaptation)};
  const cudaError_t err = nsb::launch_event_rows(
      t, e, o, to_out(*out_emitted), exchange ? &px : nullptr,
      static_cast<nsb::EventRowsState*>(workspace), static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, name);
  return NSB_OK;
}
}  // namespace

int nsb_dendritic_event_rows(const nsb_tick* tick, const nsb_event_rows* ev, float* delta,
                             const nsb_delta_exchange* exchange, const nsb_tick_out* out,
                             const nsb_out* out_emitted, void* workspace, void* stream) {
  return event_rows(tick, ev, delta, exchange, nullptr, out, out_emitted, workspace, stream,
                    "nsb_dendritic_event_rows launch");
}

int nsb_dendritic_event_rows_gated(const nsb_tick* tick, const nsb_event_rows* ev,
                                   const nsb_delta_exchange* exchange, const int32_t* out_degree,
                                   const nsb_tick_out* out, const nsb_out* out_emitted,
                                   void* workspace, void* stream) {
  if (!tick || tick->batch != 1) return fail(NSB_ERR_ARGUMENT, "the gated row tick takes B = 1");
  if (!exchange) return fail(NSB_ERR_ARGUMENT, "the gated row tick needs a peer exchange");
  if (!out_degree) return fail(NSB_ERR_ARGUMENT, "the gated row tick needs the rows' out-degrees");
  return event_rows(tick, ev, nullptr, exchange, out_degree, out, out_emitted, workspace, stream,
                    "nsb_dendritic_event_rows_gated launch");
}

int nsb_event_scatter_rows(int64_t batch, int64_t neurons, int64_t rows, const float* delta,
                           const nsb_scatter_rows* csr, float* current,
                           const nsb_delta_exchange* exchange, void* workspace, int* status,
                           void* stream) {
  if (batch < 0 || neurons <= 0 || rows < 0 || rows > neurons || batch * neurons >= (int64_t(1) << 40))
    return fail(NSB_ERR_ARGUMENT, "scatter geometry: B >= 0, N > 0, 0 <= rows <= N");
  if (!csr || !csr->rowptr || csr->n_edges < 0 || csr->n_edges >= (int64_t(1) << 31) ||
      (csr->n_edges > 0 && (!csr->dst || !csr->weight)))
    return fail(NSB_ERR_ARGUMENT, "invalid row-scatter topology geometry");
  if (batch > 0 && rows > 0 && !current) return fail(NSB_ERR_ARGUMENT, "current is required");
  if (!exchange && !delta) return fail(NSB_ERR_ARGUMENT, "a delta buffer or an exchange is required");
  nsb::DeltaPeers px{};
  if (exchange && !check_delta_exchange(exchange, &px)) return NSB_ERR_ARGUMENT;
  if (!check_rows_workspace(workspace)) return NSB_ERR_WORKSPACE;
  g_error.clear();
  if (batch == 0) return NSB_OK;
  const nsb::ScatterRowsArgs c{csr->rowptr, csr->dst, csr->weight, csr->n_edges};
  const cudaError_t err = nsb::launch_event_scatter_rows(
      batch, neurons, rows, delta, c, current, exchange ? &px : nullptr,
      static_cast<nsb::EventRowsState*>(workspace), status,
      static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_event_scatter_rows launch");
  return NSB_OK;
}

int nsb_event_scatter_rows_gated(int64_t neurons, int64_t rows, const nsb_scatter_rows* csr,
                                 float* current, const nsb_delta_exchange* exchange,
                                 uint64_t gate_edges, void* workspace, int* status, void* stream) {
  if (neurons <= 0 || rows < 0 || rows > neurons || neurons >= (int64_t(1) << 40))
    return fail(NSB_ERR_ARGUMENT, "scatter geometry: N > 0, 0 <= rows <= N");
  if (!csr || !csr->rowptr || csr->n_edges < 0 || csr->n_edges >= (int64_t(1) << 31) ||
      (csr->n_edges > 0 && (!csr->dst || !csr->weight)))
    return fail(NSB_ERR_ARGUMENT, "invalid row-scatter topology geometry");
  if (rows > 0 && !current) return fail(NSB_ERR_ARGUMENT, "current is required");
  if (!exchange) return fail(NSB_ERR_ARGUMENT, "the gated scatter needs a peer exchange");
  if (gate_edges < 1) return fail(NSB_ERR_ARGUMENT, "gate_edges must be at least 1");
  nsb::DeltaPeers px{};
  if (!check_delta_exchange(exchange, &px)) return NSB_ERR_ARGUMENT;
  if (!check_rows_workspace(workspace)) return NSB_ERR_WORKSPACE;
  g_error.clear();
  const nsb::ScatterRowsArgs c{csr->rowptr, csr->dst, csr->weight, csr->n_edges};
  const cudaError_t err = nsb::launch_event_scatter_rows(
      1, neurons, rows, nullptr, c, current, &px, static_cast<nsb::EventRowsState*>(workspace),
      status, static_cast<cudaStream_t>(stream), gate_edges);
  if (err != cudaSuccess) return cuda_fail(err, "nsb_event_scatter_rows_gated launch");
  return NSB_OK;
}

int nsb_tiled_propagate_rows_gated(const nsb_tiled_layout* layout, void* tiled_workspace,
                                   size_t tiled_workspace_bytes, float* current,
                                   uint64_t gate_edges, void* workspace, int* status,
                                   void* stream) {
  if (!check_tiled(layout)) return tiled_status(NSB_ERR_ARGUMENT);
  if (layout->format != NSB_WEIGHT_F32)
    return fail(NSB_ERR_ARGUMENT, "the gated propagate takes a float32 layout");
  if (!check_workspace(layout, tiled_workspace, tiled_workspace_bytes))
    return tiled_status(NSB_ERR_WORKSPACE);
  if (!current) return fail(NSB_ERR_ARGUMENT, "current is required");
  if (gate_edges < 1) return fail(NSB_ERR_ARGUMENT, "gate_edges must be at least 1");
  if (!check_rows_workspace(workspace)) return NSB_ERR_WORKSPACE;
  g_error.clear();
  const auto* state = static_cast<const nsb::EventRowsState*>(workspace);
  nsb::TiledGate gate;
  gate.count = &state->gate_count;
  gate.min = gate_edges;
  gate.accumulate = true;
  gate.source = &state->gate_source;
  nsb::TickArgs none{};
  none.batch = 1;
  none.neurons = layout->rows;
  const cudaError_t err = nsb::launch_tiled(*layout, none, current, false, 1, nsb::TickOut{},
                                            nsb::Out{current, 0, 1}, tiled_workspace, status,
                                            static_cast<cudaStream_t>(stream), nullptr, gate);
  if (err != cudaSuccess) return cuda_fail(err, "nsb_tiled_propagate_rows_gated launch");
  return NSB_OK;
}

int nsb_encode_weights(int32_t format, const float* weight, int64_t n, uint8_t* codes,
                       uint8_t* block_scales, float* global_scale, void* workspace,
                       void* stream) {
  if (format != NSB_WEIGHT_E4M3 && format != NSB_WEIGHT_NVFP4)
    return fail(NSB_ERR_ARGUMENT, "the encoder takes NSB_WEIGHT_E4M3 or NSB_WEIGHT_NVFP4");
  if (n < 0 || n >= (int64_t(1) << 31))
    return fail(NSB_ERR_ARGUMENT, "weight count must be in [0, 2^31)");
  if (n > 0 && (!weight || !codes))
    return fail(NSB_ERR_ARGUMENT, "weights and a code buffer are required");
  if (n > 0 && format == NSB_WEIGHT_NVFP4 && !block_scales)
    return fail(NSB_ERR_ARGUMENT, "NVFP4 encoding needs a block-scale buffer");
  if (!global_scale) return fail(NSB_ERR_ARGUMENT, "a global-scale output is required");
  if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 4 != 0)
    return fail(NSB_ERR_WORKSPACE, "encoder workspace must be 4-byte aligned");
  g_error.clear();
  const cudaError_t err = nsb::launch_encode(format, weight, n, codes, block_scales, global_scale,
                                             workspace, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "nsb_encode_weights launch");
  return NSB_OK;
}

int nsb_dendritic_event_noalloc(const nsb_tick* tick, float* current, const nsb_view* emitted,
                                const float* theta, int64_t theta_stride,
                                const nsb_out_csr* out_csr, const nsb_tick_out* out,
                                const nsb_out* out_emitted, void* stream) {
  if (tick && tick->batch > 0 && tick->neurons > 0 &&
      tick->batch * tick->neurons > static_cast<int64_t>(NSB_EVENT_NOALLOC_MAX_PAIRS))
    return fail(NSB_ERR_ARGUMENT,
                "nsb_dendritic_event_noalloc: B*N = " + std::to_string(tick->batch * tick->neurons) +
                    " exceeds its fixed scratch of " + std::to_string(NSB_EVENT_NOALLOC_MAX_PAIRS) +
                    " pairs; use nsb_dendritic_event with a caller workspace");
  void* scratch = nullptr;
  const cudaError_t err = nsb::event_noalloc_scratch(&scratch);
  if (err != cudaSuccess) return cuda_fail(err, "nsb_dendritic_event_noalloc scratch address");
  return nsb_dendritic_event(tick, current, emitted, theta, theta_stride, out_csr, out,
                             out_emitted, scratch,
                             nsb::event_workspace_bytes(tick ? tick->batch : 0,
                                                        tick ? tick->neurons : 0),
                             stream);
}

}  // extern "C"
