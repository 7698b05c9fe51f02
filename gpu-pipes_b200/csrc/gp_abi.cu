// C ABI of libgpipes.so: argument validation, per-device state, TMA descriptor creation and
// dispatch of a layer chain to a compiled fused-chain kernel.
//
// Reference boundary being replaced: the per-app pybind11 wrappers
// apps/<app>/pipelined/<app>_pl_ext.cu (e.g. apps/mgn_fullmlp/pipelined/mgn_fullmlp_pl_ext.cu:24-93),
// which assert widths, lazily allocate a process-static queue scratch (global_queue_space(),
// apps/mgn_fullmlp/pipelined/mgn_fullmlp_pl.cuh:255-266) and launch on the legacy default stream.
// Here: widths are runtime-checked against compiled instantiations, errors are returned (never
// abort), state is per device (created under a mutex), the kernels need no global scratch at all,
// and the launch goes to the caller's stream.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gpipes.h"
#include "chain_common.cuh"
#include "chain_registry.h"

namespace gp {

// ------------------------------------------------------------------------------------------------
// errors
// ------------------------------------------------------------------------------------------------
static thread_local std::string t_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

void clear_error() { t_last_error.clear(); }

// ------------------------------------------------------------------------------------------------
// global knobs
// ------------------------------------------------------------------------------------------------
static std::atomic<unsigned long long> g_timeout_ns{2000000000ull};
static std::atomic<int> g_inject{0};
static std::atomic<uint64_t> g_launches{0};

unsigned long long current_timeout_ns() { return g_timeout_ns.load(); }
int current_fault_injection() { return g_inject.load(); }
void count_launches(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

static bool sync_check_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GP_SYNC_CHECK");
    return e != nullptr && e[0] == '1';
  }();
  return on;
}

// ------------------------------------------------------------------------------------------------
// per-device state
// ------------------------------------------------------------------------------------------------
struct DeviceState {
  int sm_count = 0;
  int* status = nullptr;  // device status word
};

static std::mutex g_mu;
static std::vector<DeviceState*> g_states;
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if (static_cast<int>(g_states.size()) <= dev) g_states.resize(dev + 1, nullptr);
  if (g_states[dev] == nullptr) {
    auto* st = new DeviceState();
    e = cudaDeviceGetAttribute(&st->sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      delete st;
      return set_error(GP_ERR_CUDA, "device attribute: %s", cudaGetErrorString(e));
    }
    e = cudaMalloc(&st->status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(st->status, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      delete st;
      return set_error(GP_ERR_CUDA, "status word: %s", cudaGetErrorString(e));
    }
    g_states[dev] = st;
  }
  *out = g_states[dev];
  return GP_OK;
}

// 2-D tensor map over a row-major [rows, cols] 16-bit matrix, box [box_rows, box_cols], the given
// swizzle, zero fill outside the tensor.
// Encoded tensor maps, cached per host thread: a call on the same buffers and shapes as a recent
// one (the common case for a serving loop or a benchmark) skips cuTensorMapEncodeTiled, which
// is a few microseconds of host time per map. The descriptor depends only on its arguments.
namespace {
struct TmapKey {
  uint64_t v[8];
  bool operator==(const TmapKey& o) const { return std::memcmp(v, o.v, sizeof(v)) == 0; }
};
struct TmapSlot {
  TmapKey key;
  CUtensorMap map;
  bool used = false;
};
constexpr int kTmapCacheSlots = 64;
thread_local TmapSlot t_tmaps[kTmapCacheSlots];

TmapSlot& tmap_slot(const TmapKey& k) {
  uint64_t h = 1469598103934665603ull;
  for (uint64_t x : k.v) h = (h ^ x) * 1099511628211ull;
  return t_tmaps[(h >> 17) % kTmapCacheSlots];
}
}  // namespace

int make_tmap_2d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                 uint32_t box_cols, uint32_t box_rows, int swizzle_bytes, uint64_t ld) {
  const TmapKey key{{reinterpret_cast<uint64_t>(base), static_cast<uint64_t>(dtype), rows, cols,
                     (static_cast<uint64_t>(box_cols) << 32) | box_rows, static_cast<uint64_t>(swizzle_bytes),
                     ld, 2}};
  TmapSlot& slot = tmap_slot(key);
  if (slot.used && slot.key == key) {
    std::memcpy(map, &slot.map, sizeof(CUtensorMap));
    return GP_OK;
  }
  const CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                                      : CU_TENSOR_MAP_SWIZZLE_NONE;
  const CUtensorMapDataType dt =
      dtype == GP_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {(ld != 0 ? ld : cols) * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled failed (%d) rows=%llu cols=%llu", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols);
  slot.key = key;
  std::memcpy(&slot.map, map, sizeof(CUtensorMap));
  slot.used = true;
  return GP_OK;
}

// fp32 matrix [rows, cols] (row-major) with box {box_cols, box_rows}
int make_tmap_2d_f32(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                     uint32_t box_rows, int swizzle_bytes) {
  const CUtensorMapSwizzle sw = swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled (fp32) failed (%d) rows=%llu cols=%llu", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols);
  return GP_OK;
}

// Weight matrix [rows = K, cols = N] (row-major, 16-bit) as a 3-D map {64, K, N / 64} with the
// 64-column blocks 128 bytes apart; box {64, box_rows, box_blocks}, SWIZZLE_128B.
int make_tmap_w3d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                  uint32_t box_rows, uint32_t box_blocks) {
  if (cols % 64 != 0)
    return set_error(GP_ERR_SHAPE, "weight width %llu is not a multiple of 64", (unsigned long long)cols);
  const TmapKey key{{reinterpret_cast<uint64_t>(base), static_cast<uint64_t>(dtype), rows, cols,
                     (static_cast<uint64_t>(box_rows) << 32) | box_blocks, 0, 0, 3}};
  TmapSlot& slot = tmap_slot(key);
  if (slot.used && slot.key == key) {
    std::memcpy(map, &slot.map, sizeof(CUtensorMap));
    return GP_OK;
  }
  const CUtensorMapDataType dt =
      dtype == GP_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {cols * 2, 128};
  cuuint32_t box[3] = {64, box_rows, box_blocks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled (3-D) failed (%d) rows=%llu cols=%llu", (int)r,
                     (unsigned long long)rows, (unsigned long long)cols);
  slot.key = key;
  std::memcpy(&slot.map, map, sizeof(CUtensorMap));
  slot.used = true;
  return GP_OK;
}

// ------------------------------------------------------------------------------------------------
// per-device workspace
// ------------------------------------------------------------------------------------------------
struct Workspace {
  std::mutex mu;
  void* ptr = nullptr;
  size_t size = 0;
  cudaEvent_t last_use = nullptr;  // recorded after the latest user's launches
  bool capturing = false;          // the current holder is recording a CUDA graph
};
static Workspace g_ws[64];

int workspace_acquire(size_t bytes, cudaStream_t stream, void** ptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return set_error(GP_ERR_ARG, "device %d out of range", dev);
  Workspace& w = g_ws[dev];
  w.mu.lock();
  if (w.last_use == nullptr) {
    e = cudaEventCreateWithFlags(&w.last_use, cudaEventDisableTiming);
    if (e != cudaSuccess) {
      w.mu.unlock();
      return set_error(GP_ERR_CUDA, "workspace event: %s", cudaGetErrorString(e));
    }
  }
  // Under stream capture (a CUDA graph being recorded) the buffer is neither grown nor ordered
  // through last_use: a captured node may not wait on uncaptured work, and an event recorded in
  // the capture would not describe the replays. The graph's replays are ordered by the stream they
  // are launched on; eager calls on other streams must not overlap them.
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) {
    w.mu.unlock();
    return set_error(GP_ERR_CUDA, "cudaStreamIsCapturing: %s", cudaGetErrorString(e));
  }
  w.capturing = cap != cudaStreamCaptureStatusNone;
  if (w.capturing) {
    if (w.size < bytes) {
      w.mu.unlock();
      return set_error(GP_ERR_UNSUPPORTED,
                       "workspace of %zu bytes needed during stream capture (have %zu): run the call "
                       "once outside the capture first", bytes, w.size);
    }
    *ptr = w.ptr;
    return GP_OK;
  }
  if (w.size < bytes) {
    // growing: earlier users must be done with the old buffer
    e = cudaEventSynchronize(w.last_use);
    if (e == cudaSuccess && w.ptr != nullptr) e = cudaFree(w.ptr);
    w.ptr = nullptr;
    w.size = 0;
    const size_t grown = ((bytes + (size_t(1) << 20) - 1) >> 20) << 20;
    if (e == cudaSuccess) e = cudaMalloc(&w.ptr, grown);
    if (e != cudaSuccess) {
      w.mu.unlock();
      return set_error(GP_ERR_CUDA, "workspace of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    w.size = grown;
  }
  e = cudaStreamWaitEvent(stream, w.last_use, 0);
  if (e != cudaSuccess) {
    w.mu.unlock();
    return set_error(GP_ERR_CUDA, "workspace ordering: %s", cudaGetErrorString(e));
  }
  *ptr = w.ptr;
  return GP_OK;
}

void workspace_release(cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  Workspace& w = g_ws[dev];
  if (!w.capturing) cudaEventRecord(w.last_use, stream);
  w.capturing = false;
  w.mu.unlock();
}

static bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static int validate(const gp_mlp_spec* spec, int64_t m, const void* x, const void* const* w,
                    const void* const* b, const void* gamma, const void* beta, const void* out) {
  if (spec == nullptr) return set_error(GP_ERR_ARG, "spec is NULL");
  if (spec->n_layers < 1 || spec->n_layers > GP_MAX_LAYERS)
    return set_error(GP_ERR_SHAPE, "n_layers %d out of range [1, %d]", spec->n_layers, GP_MAX_LAYERS);
  if (spec->dtype != GP_F16 && spec->dtype != GP_BF16)
    return set_error(GP_ERR_ARG, "dtype %d unknown", spec->dtype);
  if (m < 0) return set_error(GP_ERR_ARG, "m = %lld is negative", (long long)m);
  if (m >= (int64_t(1) << 31)) return set_error(GP_ERR_SHAPE, "m = %lld exceeds 2^31-1", (long long)m);
  for (int l = 0; l <= spec->n_layers; ++l)
    if (spec->widths[l] <= 0)
      return set_error(GP_ERR_SHAPE, "width[%d] = %d must be positive", l, spec->widths[l]);
  if (spec->widths[0] % 8 != 0)
    return set_error(GP_ERR_SHAPE, "input width %d must be a multiple of 8 (16-byte rows)", spec->widths[0]);
  if (spec->skip_layer < 0 || spec->skip_layer >= spec->n_layers)
    return set_error(GP_ERR_SHAPE, "skip_layer %d out of range [0, %d)", spec->skip_layer, spec->n_layers);
  if (x == nullptr || out == nullptr || w == nullptr)
    return set_error(GP_ERR_ARG, "x, w and out must not be NULL");
  if (!aligned(x, 16) || !aligned(out, 16))
    return set_error(GP_ERR_ALIGN, "x and out must be 16-byte aligned");
  for (int l = 0; l < spec->n_layers; ++l) {
    if (w[l] == nullptr) return set_error(GP_ERR_ARG, "w[%d] is NULL", l);
    if (!aligned(w[l], 16)) return set_error(GP_ERR_ALIGN, "w[%d] must be 16-byte aligned", l);
    if (b != nullptr && b[l] != nullptr && !aligned(b[l], 4))
      return set_error(GP_ERR_ALIGN, "b[%d] must be 4-byte aligned", l);
  }
  if ((gamma != nullptr && !aligned(gamma, 4)) || (beta != nullptr && !aligned(beta, 4)))
    return set_error(GP_ERR_ALIGN, "gamma and beta must be 4-byte aligned");
  if (spec->tail < GP_TAIL_NONE || spec->tail > GP_TAIL_RESIDUAL_LN)
    return set_error(GP_ERR_ARG, "tail %d unknown", spec->tail);
  if (spec->tail == GP_TAIL_RESIDUAL_LN && spec->widths[0] != spec->widths[spec->n_layers])
    return set_error(GP_ERR_SHAPE, "residual tail needs K0 == N_last (%d vs %d)", spec->widths[0],
                     spec->widths[spec->n_layers]);
  return GP_OK;
}

int finish_launch(cudaStream_t stream, int dev_status_check) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  if (dev_status_check && sync_check_enabled()) {
    e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "sync: %s", cudaGetErrorString(e));
    DeviceState* st = nullptr;
    int rc = get_device_state(&st);
    if (rc != GP_OK) return rc;
    int h = 0;
    e = cudaMemcpy(&h, st->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
    if (h != 0) return set_error(GP_ERR_TIMEOUT, "device wait ran out (status 0x%x)", h);
  }
  return GP_OK;
}

// resid: residual rows of a GP_TAIL_RESIDUAL_LN chain ([m, N_last]); null means x itself.
int fused_mlp(const gp_mlp_spec* spec, int64_t m, const void* x, const void* const* w,
              const void* const* b, const void* gamma, const void* beta, void* out,
              cudaStream_t stream, const void* resid = nullptr) {
  clear_error();
  int rc = validate(spec, m, x, w, b, gamma, beta, out);
  if (rc != GP_OK) return rc;
  const ChainEntry* ent = find_chain(*spec);
  if (ent == nullptr) {
    std::string desc;
    for (int l = 0; l <= spec->n_layers; ++l) desc += std::to_string(spec->widths[l]) + (l < spec->n_layers ? "->" : "");
    return set_error(GP_ERR_UNSUPPORTED, "no compiled kernel for chain %s (dtype %d, tail %d)",
                     desc.c_str(), spec->dtype, spec->tail);
  }
  if (m == 0) return GP_OK;
  DeviceState* st = nullptr;
  rc = get_device_state(&st);
  if (rc != GP_OK) return rc;

  LaunchCtx c{};
  c.spec = spec;
  c.m = m;
  c.x = x;
  c.out = out;
  c.stream = stream;
  c.sm_count = st->sm_count;
  c.args.m = m;
  c.args.num_tiles = static_cast<int>((m + kBM - 1) / kBM);
  for (int l = 0; l < spec->n_layers; ++l) {
    c.w[l] = w[l];
    c.args.bias[l] = b != nullptr ? b[l] : nullptr;
  }
  c.args.gamma = gamma;
  c.args.beta = beta;
  c.args.resid = resid != nullptr ? resid : x;
  c.args.out = out;
  c.args.ln_eps = spec->ln_eps;
  c.args.status = st->status;
  c.args.timeout_ns = g_timeout_ns.load();
  c.args.inject = g_inject.load();
  rc = ent->launch(c);
  if (rc != GP_OK) return rc;
  return finish_launch(stream, 1);
}

// ------------------------------------------------------------------------------------------------
// Host-buffer pipeline (gp_fused_mlp_host): per device, an H2D and a D2H stream, double-buffered
// device staging for x and out chunks (its own allocation, apart from the kernels' workspace, since
// chains use that inside a call), and the events that order them against the caller's stream.
// ------------------------------------------------------------------------------------------------
struct HostPipe {
  std::mutex mu;
  cudaStream_t h2d = nullptr, d2h = nullptr;
  cudaEvent_t start = nullptr, done = nullptr, x_ready[2] = {}, k_done[2] = {}, out_free[2] = {};
  void* buf = nullptr;
  size_t cap = 0;
  bool used = false;
};
static std::vector<HostPipe*> g_pipes;

static int get_host_pipe(HostPipe** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_mu);
  if (static_cast<int>(g_pipes.size()) <= dev) g_pipes.resize(dev + 1, nullptr);
  if (g_pipes[dev] == nullptr) {
    HostPipe* p = new HostPipe();
    e = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking);
    cudaEvent_t* evs[8] = {&p->start, &p->done, &p->x_ready[0], &p->x_ready[1], &p->k_done[0],
                           &p->k_done[1], &p->out_free[0], &p->out_free[1]};
    for (int i = 0; e == cudaSuccess && i < 8; ++i) e = cudaEventCreateWithFlags(evs[i], cudaEventDisableTiming);
    if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "host pipeline setup: %s", cudaGetErrorString(e));
    g_pipes[dev] = p;
  }
  *out = g_pipes[dev];
  return GP_OK;
}

int fused_mlp_host(const gp_mlp_spec* spec, int64_t m, const void* x_host, const void* const* w,
                   const void* const* b, const void* gamma, const void* beta, void* out_host,
                   int64_t chunk_rows, cudaStream_t cs) {
  clear_error();
  if (spec == nullptr) return set_error(GP_ERR_ARG, "spec is NULL");
  if (m < 0) return set_error(GP_ERR_ARG, "m = %lld is negative", (long long)m);
  if (m == 0) return GP_OK;
  if (x_host == nullptr || out_host == nullptr) return set_error(GP_ERR_ARG, "x_host and out_host must not be NULL");
  if (spec->n_layers < 1 || spec->n_layers > GP_MAX_LAYERS) return set_error(GP_ERR_ARG, "n_layers = %d", spec->n_layers);
  const size_t xrow = static_cast<size_t>(spec->widths[0]) * 2;
  const size_t orow = static_cast<size_t>(spec->widths[spec->n_layers]) * 2;
  if (chunk_rows <= 0) {
    // about 16 MB of rows (x + out) per chunk and at least eight chunks, so the first upload and
    // the last download, which nothing overlaps, stay short; at least 4,096 rows, below which
    // the per-chunk launch and copy costs dominate. Measured end to end (MGN node, 1,048,576
    // rows: 9.7e7 rows/s with 131,072-row chunks, 1.02e8 with 32,768; MGN edge, 65,536 rows in
    // one chunk: 4.8e7, in 8,192-row chunks 6.4e7).
    const int64_t by_bytes = static_cast<int64_t>((size_t(16) << 20) / (xrow + orow));
    chunk_rows = (m + 7) / 8;
    if (chunk_rows > by_bytes) chunk_rows = by_bytes;
    if (chunk_rows < 4096) chunk_rows = 4096;
  }
  chunk_rows = (chunk_rows + 255) / 256 * 256;
  if (chunk_rows > m) chunk_rows = m;
  HostPipe* hp = nullptr;
  int rc = get_host_pipe(&hp);
  if (rc != GP_OK) return rc;
  std::lock_guard<std::mutex> lk(hp->mu);
  const size_t xb = (static_cast<size_t>(chunk_rows) * xrow + 255) / 256 * 256;
  const size_t ob = (static_cast<size_t>(chunk_rows) * orow + 255) / 256 * 256;
  cudaError_t e = cudaSuccess;
  if (2 * (xb + ob) > hp->cap) {
    if (hp->buf != nullptr) {
      e = cudaDeviceSynchronize();  // the previous staging may still be in use on any stream
      if (e == cudaSuccess) e = cudaFree(hp->buf);
      hp->buf = nullptr;
      hp->cap = 0;
    }
    if (e == cudaSuccess) e = cudaMalloc(&hp->buf, 2 * (xb + ob));
    if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "host pipeline staging (%zu bytes): %s", 2 * (xb + ob), cudaGetErrorString(e));
    hp->cap = 2 * (xb + ob);
  }
  char* base = static_cast<char*>(hp->buf);
  char* xbuf[2] = {base, base + xb};
  char* obuf[2] = {base + 2 * xb, base + 2 * xb + ob};
  auto ck = [&](cudaError_t r) { if (e == cudaSuccess) e = r; };
  // the copies start after the caller's earlier work, and after the previous call's last copy
  ck(cudaEventRecord(hp->start, cs));
  ck(cudaStreamWaitEvent(hp->h2d, hp->start, 0));
  if (hp->used) ck(cudaStreamWaitEvent(hp->h2d, hp->done, 0));
  const int64_t nchunks = (m + chunk_rows - 1) / chunk_rows;
  for (int64_t i = 0; rc == GP_OK && e == cudaSuccess && i < nchunks; ++i) {
    const int s = static_cast<int>(i & 1);
    const int64_t r0 = i * chunk_rows;
    const int64_t rows = (m - r0) < chunk_rows ? (m - r0) : chunk_rows;
    if (i >= 2) ck(cudaStreamWaitEvent(hp->h2d, hp->k_done[s], 0));  // chunk i-2 has read xbuf[s]
    ck(cudaMemcpyAsync(xbuf[s], static_cast<const char*>(x_host) + r0 * xrow, rows * xrow,
                       cudaMemcpyHostToDevice, hp->h2d));
    ck(cudaEventRecord(hp->x_ready[s], hp->h2d));
    ck(cudaStreamWaitEvent(cs, hp->x_ready[s], 0));
    if (i >= 2) ck(cudaStreamWaitEvent(cs, hp->out_free[s], 0));  // chunk i-2's D2H has read obuf[s]
    if (e != cudaSuccess) break;
    rc = fused_mlp(spec, rows, xbuf[s], w, b, gamma, beta, obuf[s], cs);
    ck(cudaEventRecord(hp->k_done[s], cs));
    ck(cudaStreamWaitEvent(hp->d2h, hp->k_done[s], 0));
    ck(cudaMemcpyAsync(static_cast<char*>(out_host) + r0 * orow, obuf[s], rows * orow,
                       cudaMemcpyDeviceToHost, hp->d2h));
    ck(cudaEventRecord(hp->out_free[s], hp->d2h));
  }
  // the caller's stream (and the next call) see every copy finished
  ck(cudaEventRecord(hp->done, hp->d2h));
  ck(cudaStreamWaitEvent(cs, hp->done, 0));
  hp->used = true;
  if (rc != GP_OK) return rc;
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "host pipeline: %s", cudaGetErrorString(e));
  return GP_OK;
}

}  // namespace gp

// ================================================================================================
// extern "C"
// ================================================================================================
using namespace gp;

extern "C" {

int gp_fused_mlp_out(const gp_mlp_spec* spec, int64_t m, const void* x, const void* const* w,
                     const void* const* b, const void* gamma, const void* beta, void* out,
                     void* stream) {
  return fused_mlp(spec, m, x, w, b, gamma, beta, out, static_cast<cudaStream_t>(stream));
}

int gp_fused_mlp_host(const gp_mlp_spec* spec, int64_t m, const void* x_host, const void* const* w,
                      const void* const* b, const void* gamma, const void* beta, void* out_host,
                      int64_t chunk_rows, void* stream) {
  return fused_mlp_host(spec, m, x_host, w, b, gamma, beta, out_host, chunk_rows,
                        static_cast<cudaStream_t>(stream));
}

static gp_mlp_spec mgn_spec(int k0, int tail, int dtype) {
  gp_mlp_spec s{};
  s.n_layers = 3;
  s.widths[0] = k0;
  s.widths[1] = s.widths[2] = s.widths[3] = 128;
  s.act[0] = GP_ACT_RELU;
  s.act[1] = GP_ACT_RELU;
  s.act[2] = GP_ACT_NONE;
  s.tail = tail;
  s.dtype = dtype;
  s.ln_eps = 1e-5f;
  return s;
}

int gp_mgn_fullmlp_out(int64_t m, int k0, const void* x, const void* w1, const void* b1,
                       const void* w2, const void* b2, const void* w3, const void* b3,
                       const void* gamma, const void* beta, void* out, void* stream) {
  gp_mlp_spec s = mgn_spec(k0, GP_TAIL_LAYERNORM, GP_F16);
  const void* w[3] = {w1, w2, w3};
  const void* b[3] = {b1, b2, b3};
  return fused_mlp(&s, m, x, w, b, gamma, beta, out, static_cast<cudaStream_t>(stream));
}

int gp_mgn_linears_out(int64_t m, int k0, const void* x, const void* w1, const void* b1,
                       const void* w2, const void* b2, const void* w3, const void* b3, void* out,
                       void* stream) {
  gp_mlp_spec s = mgn_spec(k0, GP_TAIL_NONE, GP_F16);
  const void* w[3] = {w1, w2, w3};
  const void* b[3] = {b1, b2, b3};
  return fused_mlp(&s, m, x, w, b, nullptr, nullptr, out, static_cast<cudaStream_t>(stream));
}

int gp_dlrm_botmlp_out(int64_t m, int k0, const void* x, const void* w1, const void* b1,
                       const void* w2, const void* b2, const void* w3, const void* b3, void* out,
                       void* stream) {
  gp_mlp_spec s{};
  s.n_layers = 3;
  const int wd[4] = {k0, 512, 256, 128};
  for (int i = 0; i < 4; ++i) s.widths[i] = wd[i];
  for (int i = 0; i < 3; ++i) s.act[i] = GP_ACT_RELU;
  s.tail = GP_TAIL_NONE;
  s.dtype = GP_F16;
  const void* w[3] = {w1, w2, w3};
  const void* b[3] = {b1, b2, b3};
  return fused_mlp(&s, m, x, w, b, nullptr, nullptr, out, static_cast<cudaStream_t>(stream));
}

static int gc_mlp(int64_t m, int k0, int dtype, int act, const void* x, const void* w0,
                  const void* b0, const void* w1, const void* b1, const void* gamma,
                  const void* beta, void* out, void* stream) {
  gp_mlp_spec s{};
  s.n_layers = 2;
  s.widths[0] = k0;
  s.widths[1] = s.widths[2] = 512;
  s.act[0] = act;
  s.act[1] = GP_ACT_NONE;
  s.tail = GP_TAIL_LAYERNORM;
  s.dtype = dtype;
  s.ln_eps = 1e-5f;
  const void* w[2] = {w0, w1};
  const void* b[2] = {b0, b1};
  return fused_mlp(&s, m, x, w, b, gamma, beta, out, static_cast<cudaStream_t>(stream));
}

int gp_gc_edges_out(int64_t m, int dtype, int act, const void* x, const void* w0, const void* b0,
                    const void* w1, const void* b1, const void* gamma, const void* beta, void* out,
                    void* stream) {
  return gc_mlp(m, 1536, dtype, act, x, w0, b0, w1, b1, gamma, beta, out, stream);
}

int gp_gc_nodes_out(int64_t m, int dtype, int act, const void* x, const void* w0, const void* b0,
                    const void* w1, const void* b1, const void* gamma, const void* beta, void* out,
                    void* stream) {
  return gc_mlp(m, 1024, dtype, act, x, w0, b0, w1, b1, gamma, beta, out, stream);
}

int gp_bert_ffn_out(int64_t m, const void* x, const void* w1, const void* b1, const void* w2,
                    const void* b2, const void* gamma, const void* beta, float ln_eps, void* out,
                    void* stream) {
  gp_mlp_spec s{};
  s.n_layers = 2;
  s.widths[0] = 1024;
  s.widths[1] = 4096;
  s.widths[2] = 1024;
  s.act[0] = GP_ACT_GELU_TANH;
  s.act[1] = GP_ACT_NONE;
  s.tail = GP_TAIL_RESIDUAL_LN;
  s.dtype = GP_BF16;
  s.ln_eps = ln_eps;
  const void* w[2] = {w1, w2};
  const void* b[2] = {b1, b2};
  return fused_mlp(&s, m, x, w, b, gamma, beta, out, static_cast<cudaStream_t>(stream));
}

int gp_dlrm_topmlp_out(int64_t m, int k0, int n_out, const void* x, const void* const* w,
                       const void* const* b, void* out, void* stream) {
  if (w == nullptr) return set_error(GP_ERR_ARG, "w is NULL");
  gp_mlp_spec s{};
  s.n_layers = 5;
  const int wd[6] = {k0, 1024, 1024, 512, 256, n_out};
  for (int i = 0; i < 6; ++i) s.widths[i] = wd[i];
  for (int i = 0; i < 4; ++i) s.act[i] = GP_ACT_RELU;
  // a single output is the click probability (sigmoid); the reference app's 64-wide output is
  // followed by DlrmMlp's ReLU
  s.act[4] = n_out == 1 ? GP_ACT_SIGMOID : GP_ACT_RELU;
  s.tail = GP_TAIL_NONE;
  s.dtype = GP_F16;
  return fused_mlp(&s, m, x, w, b, nullptr, nullptr, out, static_cast<cudaStream_t>(stream));
}

// BERT attention-output block, apps/bert_addln_ffn/pipelined/bert_addln_ffn_pl_ext.cu:15-58
// (H = 128, ff = 512, fp16): h = LN0(attn_out W0 + b0 + x), out = LN2(ReLU(h W1 + b1) W2 + b2 + h).
// Two fused chain launches; h ([m, 128] fp16) lives in the per-device workspace between them.
int gp_bert_addln_ffn_out(int64_t m, const void* attn_out, const void* x, const void* w0,
                          const void* b0, const void* w1, const void* b1, const void* w2,
                          const void* b2, const void* ga0, const void* be0, const void* ga2,
                          const void* be2, void* out, void* stream) {
  clear_error();
  if (m < 0) return set_error(GP_ERR_ARG, "m = %lld is negative", (long long)m);
  if (attn_out == nullptr || x == nullptr || out == nullptr || w0 == nullptr || w1 == nullptr ||
      w2 == nullptr)
    return set_error(GP_ERR_ARG, "attn_out, x, w0, w1, w2 and out must not be NULL");
  if (!aligned(x, 16)) return set_error(GP_ERR_ALIGN, "x must be 16-byte aligned");
  if (m == 0) return GP_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  gp_mlp_spec sa{};
  sa.n_layers = 1;
  sa.widths[0] = 128;
  sa.widths[1] = 128;
  sa.act[0] = GP_ACT_NONE;
  sa.tail = GP_TAIL_RESIDUAL_LN;
  sa.dtype = GP_F16;
  sa.ln_eps = 1e-5f;
  gp_mlp_spec sb = sa;
  sb.n_layers = 2;
  sb.widths[1] = 512;
  sb.widths[2] = 128;
  sb.act[0] = GP_ACT_RELU;
  sb.act[1] = GP_ACT_NONE;
  void* h = nullptr;
  int rc = workspace_acquire(static_cast<size_t>(m) * 128 * 2, s, &h);
  if (rc != GP_OK) return rc;
  const void* wa[1] = {w0};
  const void* ba[1] = {b0};
  rc = fused_mlp(&sa, m, attn_out, wa, ba, ga0, be0, h, s, x);
  if (rc == GP_OK) {
    const void* wb[2] = {w1, w2};
    const void* bb[2] = {b1, b2};
    rc = fused_mlp(&sb, m, h, wb, bb, ga2, be2, out, s);
  }
  workspace_release(s);
  return rc;
}

// DLRM feature interaction (graphmodel/dlrm.py:28-42): out [m, 480] = [bot | strict lower
// triangle of [bot; e_0..e_25] [bot; e_0..e_25]^T | 0], the top MLP's input. fp16.
int gp_dlrm_interaction_out(int64_t m, const void* bot, const void* sparse, void* out, void* stream) {
  clear_error();
  if (m < 0) return set_error(GP_ERR_ARG, "m = %lld is negative", (long long)m);
  if (m >= (int64_t(1) << 31)) return set_error(GP_ERR_SHAPE, "m = %lld exceeds 2^31-1", (long long)m);
  if (bot == nullptr || sparse == nullptr || out == nullptr)
    return set_error(GP_ERR_ARG, "bot, sparse and out must not be NULL");
  if (!aligned(bot, 16) || !aligned(sparse, 16) || !aligned(out, 16))
    return set_error(GP_ERR_ALIGN, "bot, sparse and out must be 16-byte aligned");
  if (m == 0) return GP_OK;
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != GP_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  rc = launch_dlrm_interaction(m, bot, sparse, out, s, st->sm_count, st->status, g_timeout_ns.load());
  if (rc != GP_OK) return rc;
  return finish_launch(s, 1);
}

static gp_mlp_spec nerf_spec(bool head) {
  gp_mlp_spec s{};
  s.n_layers = head ? 9 : 8;
  s.widths[0] = 64;
  for (int i = 1; i <= 8; ++i) s.widths[i] = 256;
  if (head) s.widths[9] = 4;
  for (int i = 0; i < 8; ++i) s.act[i] = GP_ACT_RELU;
  s.act[8] = GP_ACT_NONE;
  s.tail = GP_TAIL_NONE;
  s.dtype = GP_F16;
  s.skip_layer = 5;
  return s;
}

int gp_nerf_a_out(int64_t m, const void* x, const void* const* w, const void* const* b, void* out,
                  void* stream) {
  if (w == nullptr) return set_error(GP_ERR_ARG, "w is NULL");
  gp_mlp_spec s = nerf_spec(false);
  return fused_mlp(&s, m, x, w, b, nullptr, nullptr, out, static_cast<cudaStream_t>(stream));
}

int gp_nerf_out(int64_t m, const void* x, const void* const* w, const void* const* b, void* out,
                void* stream) {
  if (w == nullptr) return set_error(GP_ERR_ARG, "w is NULL");
  gp_mlp_spec s = nerf_spec(true);
  return fused_mlp(&s, m, x, w, b, nullptr, nullptr, out, static_cast<cudaStream_t>(stream));
}

// NeRF with view directions (apps/nerf_full/pipelined/nerf_full_pl_ext.cu:22-95), one fused chain
// kernel (trunk, alpha side output, bottleneck, [bottleneck | d] -> rgb): x [m, 64],
// d [m, 32] -> out_r [m, 64] = encoded w9 + b9, out_rgb [m, 64] = ReLU([encoded w10 + b10 | d]
// w11 + b11) w12 + b12. fp16. w[0..11] / b[0..11] are the reference's w1..w12 / b1..b12 (b may
// be NULL, or hold NULL entries).
int gp_nerf_full_out(int64_t m, const void* x, const void* d, const void* const* w,
                     const void* const* b, void* out_r, void* out_rgb, void* stream) {
  clear_error();
  if (m < 0) return set_error(GP_ERR_ARG, "m = %lld is negative", (long long)m);
  if (m >= (int64_t(1) << 31)) return set_error(GP_ERR_SHAPE, "m = %lld exceeds 2^31-1", (long long)m);
  if (m == 0) return GP_OK;
  if (x == nullptr || d == nullptr || w == nullptr || out_r == nullptr || out_rgb == nullptr)
    return set_error(GP_ERR_ARG, "x, d, w, out_r and out_rgb must not be NULL");
  const void* bb[12] = {nullptr};
  for (int i = 0; i < 12; ++i) {
    if (w[i] == nullptr) return set_error(GP_ERR_ARG, "w[%d] is NULL", i);
    if (!aligned(w[i], 16)) return set_error(GP_ERR_ALIGN, "w[%d] must be 16-byte aligned", i);
    bb[i] = b != nullptr ? b[i] : nullptr;
    if (bb[i] != nullptr && !aligned(bb[i], 16)) return set_error(GP_ERR_ALIGN, "b[%d] must be 16-byte aligned", i);
  }
  if (!aligned(x, 16) || !aligned(d, 16) || !aligned(out_r, 16) || !aligned(out_rgb, 16))
    return set_error(GP_ERR_ALIGN, "x, d, out_r and out_rgb must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != GP_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchCtx c{};
  c.stream = s;
  c.sm_count = st->sm_count;
  c.args.status = st->status;
  c.args.timeout_ns = g_timeout_ns.load();
  c.args.inject = g_inject.load();
  rc = launch_nerf_full(c, m, x, d, w, bb, out_r, out_rgb);  // one fused chain kernel
  if (rc != GP_OK) return rc;
  return finish_launch(s, 1);
}

// MeshGraphNet edge update with the gather fused (graphmodel/mgn_dp.py:28-32) and, when agg is
// set, the scatter-sum of the outputs by destination node fused into the same kernel.
int gp_mgn_edge_update_out(int64_t m, int64_t n_nodes, const void* nf, const void* ef,
                           const int64_t* srcs, const int64_t* dsts, const void* const* w,
                           const void* const* b, const void* gamma, const void* beta, void* out,
                           float* agg, void* stream) {
  clear_error();
  if (m < 0 || n_nodes < 0) return set_error(GP_ERR_ARG, "m = %lld, n_nodes = %lld", (long long)m, (long long)n_nodes);
  if (m >= (int64_t(1) << 31)) return set_error(GP_ERR_SHAPE, "m = %lld exceeds 2^31-1", (long long)m);
  if (m == 0) return GP_OK;
  if (n_nodes == 0) return set_error(GP_ERR_ARG, "edges need nodes (n_nodes = 0)");
  if (n_nodes > (int64_t(1) << 25))  // node row offsets (node * 128) are 32-bit in the kernel
    return set_error(GP_ERR_SHAPE, "n_nodes = %lld exceeds 2^25", (long long)n_nodes);
  if (nf == nullptr || ef == nullptr || srcs == nullptr || dsts == nullptr || w == nullptr || out == nullptr)
    return set_error(GP_ERR_ARG, "nf, ef, srcs, dsts, w and out must not be NULL");
  for (int l = 0; l < 3; ++l) {
    if (w[l] == nullptr || !aligned(w[l], 16)) return set_error(GP_ERR_ALIGN, "w[%d] NULL or not 16-byte aligned", l);
    if (b != nullptr && b[l] != nullptr && !aligned(b[l], 16))
      return set_error(GP_ERR_ALIGN, "b[%d] must be 16-byte aligned", l);
  }
  if (!aligned(nf, 16) || !aligned(ef, 16) || !aligned(out, 16) || !aligned(srcs, 8) || !aligned(dsts, 8) ||
      (agg != nullptr && !aligned(agg, 16)))
    return set_error(GP_ERR_ALIGN, "nf, ef, out and agg must be 16-byte aligned, srcs and dsts 8-byte");
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != GP_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchCtx c{};
  c.stream = s;
  c.sm_count = st->sm_count;
  c.args.status = st->status;
  c.args.timeout_ns = g_timeout_ns.load();
  c.args.ln_eps = 1e-5f;
  rc = launch_mgn_edge_update(c, m, n_nodes, nf, ef, srcs, dsts, w, b, gamma, beta, out, agg);
  if (rc != GP_OK) return rc;
  return finish_launch(s, 1);
}

// MeshGraphNet node update (graphmodel/mgn_dp.py:46-54) on [nf | aggregates of n_sets edge sets].
int gp_mgn_node_update_out(int64_t n, int n_sets, const void* nf, const float* const* aggs,
                           const void* const* w, const void* const* b, const void* gamma,
                           const void* beta, void* out, void* stream) {
  clear_error();
  if (n < 0) return set_error(GP_ERR_ARG, "n = %lld is negative", (long long)n);
  if (n >= (int64_t(1) << 31)) return set_error(GP_ERR_SHAPE, "n = %lld exceeds 2^31-1", (long long)n);
  if (n_sets != 1 && n_sets != 2) return set_error(GP_ERR_UNSUPPORTED, "n_sets = %d (1 or 2 edge sets)", n_sets);
  if (n == 0) return GP_OK;
  if (nf == nullptr || aggs == nullptr || w == nullptr || out == nullptr)
    return set_error(GP_ERR_ARG, "nf, aggs, w and out must not be NULL");
  for (int i = 0; i < n_sets; ++i)
    if (aggs[i] == nullptr || !aligned(aggs[i], 16)) return set_error(GP_ERR_ALIGN, "aggs[%d] NULL or not 16-byte aligned", i);
  for (int l = 0; l < 3; ++l) {
    if (w[l] == nullptr || !aligned(w[l], 16)) return set_error(GP_ERR_ALIGN, "w[%d] NULL or not 16-byte aligned", l);
    if (b != nullptr && b[l] != nullptr && !aligned(b[l], 16))
      return set_error(GP_ERR_ALIGN, "b[%d] must be 16-byte aligned", l);
  }
  if (!aligned(nf, 16) || !aligned(out, 16)) return set_error(GP_ERR_ALIGN, "nf and out must be 16-byte aligned");
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  if (rc != GP_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  LaunchCtx c{};
  c.stream = s;
  c.sm_count = st->sm_count;
  c.args.status = st->status;
  c.args.timeout_ns = g_timeout_ns.load();
  c.args.ln_eps = 1e-5f;
  rc = launch_mgn_node_update(c, n, n_sets, nf, aggs, w, b, gamma, beta, out);
  if (rc != GP_OK) return rc;
  g_launches.fetch_add(1, std::memory_order_relaxed);  // the aggregate conversion
  return finish_launch(s, 1);
}

int gp_testmlp_out(int64_t m, const void* x, const void* w1, const void* b1, const void* w2,
                   const void* b2, const void* w3, const void* b3, void* out, void* stream) {
  gp_mlp_spec s = mgn_spec(128, GP_TAIL_NONE, GP_F16);
  const void* w[3] = {w1, w2, w3};
  const void* b[3] = {b1, b2, b3};
  return fused_mlp(&s, m, x, w, b, nullptr, nullptr, out, static_cast<cudaStream_t>(stream));
}

const char* gp_last_error(void) { return t_last_error.c_str(); }

int gp_device_status(int device, int clear, int* status_out) {
  clear_error();
  int prev = 0;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  DeviceState* st = nullptr;
  int rc = get_device_state(&st);
  int h = 0;
  if (rc == GP_OK) {
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&h, st->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(st->status, 0, sizeof(int));
    if (e == cudaSuccess && clear) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) rc = set_error(GP_ERR_CUDA, "status: %s", cudaGetErrorString(e));
  }
  if (rc == GP_OK) {
    // the allocation-free entry point keeps its own status word (a file-scope device variable)
    int h_na = 0;
    rc = noalloc_status(clear != 0, &h_na);
    if (h == 0) h = h_na;
  }
  cudaSetDevice(prev);
  if (status_out != nullptr) *status_out = h;
  return rc;
}

int gp_set_timeout_ns(uint64_t ns) {
  g_timeout_ns.store(ns == 0 ? 2000000000ull : ns);
  return GP_OK;
}

int gp_set_fault_injection(int mode) {
  if (mode < 0 || mode > 1) return set_error(GP_ERR_ARG, "fault injection mode %d unknown", mode);
  g_inject.store(mode);
  return GP_OK;
}

uint64_t gp_launch_count(void) { return g_launches.load(); }

int gp_debug_pdl_flags(void* stream, int n, const void* const* ptrs, const uint64_t* bytes, const int* kinds,
                       int record) {
  clear_error();
  if (n < 0 || (n > 0 && (ptrs == nullptr || bytes == nullptr || kinds == nullptr)))
    return set_error(GP_ERR_ARG, "range arrays missing");
  for (int i = 0; i < n; ++i)
    if (kinds[i] < 0 || kinds[i] > 3) return set_error(GP_ERR_ARG, "range kind %d unknown", kinds[i]);
  return pdl_probe(static_cast<cudaStream_t>(stream), n, ptrs, bytes, kinds, record != 0);
}

int gp_set_kernel_variant(int variant) {
  if (variant < 0 || variant > 2) return set_error(GP_ERR_ARG, "kernel variant %d unknown", variant);
  set_kernel_variant(variant);
  return GP_OK;
}

}  // extern "C"
