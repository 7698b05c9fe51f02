// Registry of compiled fused-chain kernels: the host looks a gp_mlp_spec up here and calls the
// matching launcher. One entry per template instantiation.
#pragma once

#include <cuda_runtime.h>

#include "../../include/gpipes.h"
#include "chain_common.cuh"

namespace gp {

struct LaunchCtx {
  const gp_mlp_spec* spec;
  int64_t m;
  const void* x;
  void* out;
  const void* x2 = nullptr;  // second x source (resident kernel, x mode 2)
  int64_t x_ld = 0;    // row strides in elements (0 = contiguous rows); stream chains only
  int64_t out_ld = 0;
  const void* w[kMaxLayers];
  cudaStream_t stream;
  int sm_count;
  ChainArgs args;
};

using LaunchFn = int (*)(const LaunchCtx&);

struct ChainEntry {
  const char* name;
  int dtype;
  int n_layers;
  int widths[kMaxLayers + 1];
  int act[kMaxLayers];
  int tail;
  LaunchFn launch;
  int variant = 0;  // 0 = default kernel for the chain; others selectable for A/B measurements
  int skip = 0;     // skip-concat layer (gp_mlp_spec.skip_layer)
};

const ChainEntry* find_chain(const gp_mlp_spec& s);
void set_kernel_variant(int v);

// helpers implemented in gp_abi.cu
int set_error(int code, const char* fmt, ...);
void clear_error();
// swizzle_bytes: 128, 64, 32 or 0 (none)
// ld: row stride in elements (0 = cols, a contiguous matrix)
int make_tmap_2d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                 uint32_t box_cols, uint32_t box_rows, int swizzle_bytes, uint64_t ld = 0);
int make_tmap_2d_f32(CUtensorMap* map, void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
                     uint32_t box_rows, int swizzle_bytes);
// NeRF with view directions (inst_stream.cu): three chain launches sharing a workspace
int launch_nerf_full(const LaunchCtx& base, int64_t m, const void* x, const void* d,
                     const void* const* w, const void* const* b, void* out_r, void* out_rgb);
// MeshGraphNet edge and node updates (mgn_graph.cu). base carries stream, SM count, status and
// timeout. Edge: out[e] = LN(MLP([nf[src[e]] | ef[e] | nf[dst[e]]])), agg[dst[e]] += out[e] when
// agg is set. Node: out[v] = LN(MLP([nf[v] | agg_0[v] | ... ])) over n_sets fp32 aggregates.
int launch_mgn_edge_update(const LaunchCtx& base, int64_t m, int64_t n_nodes, const void* nf,
                           const void* ef, const int64_t* srcs, const int64_t* dsts,
                           const void* const* w, const void* const* b, const void* gamma,
                           const void* beta, void* out, float* agg);
int launch_mgn_node_update(const LaunchCtx& base, int64_t n, int n_sets, const void* nf,
                           const float* const* aggs, const void* const* w, const void* const* b,
                           const void* gamma, const void* beta, void* out);
// DLRM feature interaction (dlrm_interaction.cu): bot [m, 128], sparse [m, 26, 128] -> out [m, 480]
int launch_dlrm_interaction(int64_t m, const void* bot, const void* sparse, void* out,
                            cudaStream_t stream, int sm_count, int* status,
                            unsigned long long timeout_ns);
int make_tmap_w3d(CUtensorMap* map, const void* base, int dtype, uint64_t rows, uint64_t cols,
                  uint32_t box_rows, uint32_t box_blocks);

// Per-device workspace for kernels that need global scratch (fp16 weight copies, intermediates
// of multi-kernel chains). workspace_acquire returns a buffer of at least `bytes` whose earlier
// users (on any stream) are ordered before `stream`; the buffer is allocated on first use and
// grown (never shrunk) when a larger one is needed. The caller must call workspace_release on
// the same stream after enqueuing its last user; between the two calls other host threads that
// want the workspace of this device wait.
int workspace_acquire(size_t bytes, cudaStream_t stream, void** ptr);
void workspace_release(cudaStream_t stream);

// Library-wide knobs set through the C ABI (gp_abi.cu): the device wait budget, the host-side
// fault injection mode, and the launch counter behind gp_launch_count.
unsigned long long current_timeout_ns();
int current_fault_injection();
void count_launches(int n);
// Status word of the allocation-free entry point on the current device (noalloc.cu); clears it
// when `clear` is set. The caller synchronises the device first.
int noalloc_status(bool clear, int* status);

// The early-read decision and record update of one launch, without launching (diagnostics):
// kinds 0 parameter, 1 x, 2 written, 3 writes not listed. Returns the pdl_early bits.
int pdl_probe(cudaStream_t stream, int n, const void* const* ptrs, const uint64_t* bytes, const int* kinds,
              bool record);

// Sets the dynamic shared memory attribute of `kern` once per device.
int ensure_smem_attr(const void* kern, int bytes, unsigned long long* done_mask);

// Programmatic dependent launch of the persistent chain kernels (on unless the environment sets
// GP_PDL=0): a launch may start while the stream's previous kernel drains; the kernel initialises
// its barriers, then waits for that kernel (griddepcontrol.wait) before any global access.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch_chain_kernel(void (*kern)(KArgs...), int grid, int block, int smem, cudaStream_t stream,
                                Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(block), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  // a launch error is left in the runtime's last-error state, which the entry points check
  (void)cudaLaunchKernelEx(&cfg, kern, args...);
}

// Early reads under programmatic dependent launch. A chain kernel may read its weights and
// per-column parameters (bit 1 of ChainArgs::pdl_early) and its input rows (bit 2) before its
// griddepcontrol.wait, overlapping the previous kernel of the stream, when those bytes do not
// overlap anything that kernel writes. Every kernel triggers its dependents only after its own
// wait, so the previous chain kernel is the only one that can still run. PdlLaunch holds the
// per-(device, stream) record of the last chain launch's writes, under a lock kept from the flag
// computation through the launch; a stream without a record, and a launch whose writes are not
// listed exactly, allow no early reads.
struct PdlIo {
  static constexpr int kMax = 2 * kMaxLayers + 12;
  enum Kind : uint8_t { kParam = 0, kX = 1, kWrite = 2 };
  uintptr_t lo[kMax];
  uintptr_t hi[kMax];
  uint8_t kind[kMax];
  int n = 0;
  bool overflow = false;        // a range did not fit: nothing early, writes unknown
  bool writes_unknown = false;  // the next launch on the stream reads nothing early
  void add(Kind k, const void* p, uint64_t bytes) {
    if (p == nullptr || bytes == 0) return;
    if (n == kMax) {
      overflow = true;
      return;
    }
    lo[n] = reinterpret_cast<uintptr_t>(p);
    hi[n] = lo[n] + bytes;
    kind[n] = k;
    ++n;
  }
};

class PdlLaunch {
 public:
  explicit PdlLaunch(cudaStream_t stream);
  ~PdlLaunch();
  PdlLaunch(const PdlLaunch&) = delete;
  PdlLaunch& operator=(const PdlLaunch&) = delete;
  // ChainArgs::pdl_early bits allowed for a launch with these ranges
  int early_flags(const PdlIo& io) const;
  // the writes of the launch just made become the stream's record
  void record(const PdlIo& io);

 private:
  int slot_;
  bool untracked_;
};

}  // namespace gp
