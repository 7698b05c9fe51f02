// gp_gc_edges_bf16_noalloc_out: the bf16 GraphCast edge MLP without any memory allocation.
//
// Who needs this: callers that cannot allocate GPU memory at call time -- code running inside a
// framework that owns every device allocation (a custom allocator or a fixed memory budget with
// cudaMalloc forbidden), real-time or serving loops that must not enter the allocator, and
// environments where the stream-ordered pool may not be used. The regular entry point
// (gp_gc_edges_out with GP_BF16) keeps the fp16 copies of the second layer's weights in a
// per-device workspace that it allocates with cudaMalloc on first use (and grows when needed);
// this variant uses a fixed buffer compiled into the library instead:
//
//   * g_noalloc_scratch is a file-scope __device__ array of kNoAllocScratchBytes (1 MiB). Every
//     GPU that loads libgpipes.so holds it until the process exits.
//   * Host code cannot use the array's name as a device address; the first call on each device
//     (with that device current) looks the address up with cudaGetSymbolAddress and caches it.
//     That first call should therefore happen before any stream capture on that device.
//   * All calls on a device share the one buffer, and each call overwrites it completely (nothing
//     needs to start at zero). Calls whose kernels overlap on the GPU -- on different streams
//     without ordering between them -- race on the buffer; order them (one stream, or events).
//   * Chains whose converted weights exceed the buffer are rejected with GP_ERR_SHAPE.
//   * Device waits are bounded by the library's wait budget (gp_set_timeout_ns) and honour the
//     host-side fault injection (gp_set_fault_injection). A wait that runs out records its code in
//     a status word of this file -- also a file-scope __device__ variable, so reporting needs no
//     allocation either -- and the kernel exits cleanly; gp_device_status reads and clears that
//     word together with the library's own.
//   * The kernel is the single-CTA form of the weight-streaming chain kernel (the regular bf16
//     GraphCast entry point runs the CTA-pair form), so timings differ; both meet the same
//     tolerance against the fp32 model.
//
// Nothing here calls cudaMalloc, cudaMallocAsync, cudaFree or any other allocating routine.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "../../include/gpipes.h"
#include "chain_registry.h"
#include "mlp_stream.cuh"

namespace gp {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;  // 1 MiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ int g_noalloc_status;

// GraphCast edge MLP, bf16 data with fp16 hidden activations (same chain as the default kernel).
template <int ACT0>
struct ChainGcNoAlloc {
  using T = __nv_bfloat16;
  static constexpr int NL = 2;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? 1536 : 512; }
  __host__ __device__ static constexpr int N(int) { return 512; }
  __host__ __device__ static constexpr int ACT(int l) { return l == 0 ? ACT0 : kActNone; }
  static constexpr int SKIP = 0, TAIL = kTailLayerNorm, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = true;
  static constexpr int HALVES = 2;
  static constexpr bool SPLIT_ACT = false;
};

__global__ void noalloc_bf16_to_f16(const __nv_bfloat16* __restrict__ src, __half* __restrict__ dst,
                                    int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2half_rn(__bfloat162float(src[i]));
}

struct NoAllocDevice {
  bool ready = false;
  void* scratch = nullptr;   // device address of g_noalloc_scratch
  int* status = nullptr;     // device address of g_noalloc_status
  int sm_count = 0;
  bool attr_relu = false, attr_silu = false;  // guarded by g_na_mu
};

std::mutex g_na_mu;
NoAllocDevice g_na[kNoAllocMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_na_encode = nullptr;

int na_setup(int dev, NoAllocDevice** out) {
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (dev < 0 || dev >= kNoAllocMaxDevices) return set_error(GP_ERR_ARG, "device %d out of range", dev);
  if (g_na_encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e =
        cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled entry point unavailable");
    g_na_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  NoAllocDevice& d = g_na[dev];
  if (!d.ready) {
    // the device is current: resolve the device addresses of the file-scope arrays
    cudaError_t e = cudaGetSymbolAddress(&d.scratch, g_noalloc_scratch);
    if (e != cudaSuccess)
      return set_error(GP_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    void* st = nullptr;
    e = cudaGetSymbolAddress(&st, g_noalloc_status);
    if (e != cudaSuccess)
      return set_error(GP_ERR_CUDA, "cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
    d.status = static_cast<int*>(st);
    e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "device attribute: %s", cudaGetErrorString(e));
    d.ready = true;
  }
  *out = &d;
  return GP_OK;
}

int na_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t rows, uint64_t cols,
            uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle sw) {
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_na_encode(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GP_OK : set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

// weight [rows, cols] as {64, rows, cols / 64} (block stride 128 B), box {64, box_rows, box_blocks}
int na_tmap_w3d(CUtensorMap* map, const void* base, CUtensorMapDataType dt, uint64_t rows, uint64_t cols,
                uint32_t box_rows, uint32_t box_blocks) {
  cuuint64_t dims[3] = {64, rows, cols / 64};
  cuuint64_t strides[2] = {cols * 2, 128};
  cuuint32_t box[3] = {64, box_rows, box_blocks};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_na_encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? GP_OK : set_error(GP_ERR_DRIVER, "cuTensorMapEncodeTiled failed (%d)", (int)r);
}

template <int ACT0>
int na_launch(NoAllocDevice& d, int64_t m, const void* x, const void* w0, const void* b0,
              const void* w1, const void* b1, const void* gamma, const void* beta, void* out,
              cudaStream_t stream, bool* attr_done) {
  using C = ChainGcNoAlloc<ACT0>;
  using Lay = StreamLayout<C>;
  {
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!*attr_done) {
      cudaError_t e = cudaFuncSetAttribute(&mlp_stream_kernel<C>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kSmemBytes);
      if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
      *attr_done = true;
    }
  }
  // fp16 copy of the second layer's weights into the fixed buffer
  const int64_t n1 = static_cast<int64_t>(C::K(1)) * C::N(1);
  noalloc_bf16_to_f16<<<static_cast<int>((n1 + 1023) / 1024), 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(w1), static_cast<__half*>(d.scratch), n1);
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  int rc = na_tmap(&tm.x, x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, m, C::K(0), kPanel, kBM, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc == GP_OK)
    rc = na_tmap(&tm.out, out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, m, C::N(1), 32, 32, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc == GP_OK)
    rc = na_tmap_w3d(&tm.w[0], w0, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, C::K(0), C::N(0), Lay::kBK,
                     C::N(0) / Lay::NH / 64);
  if (rc == GP_OK)
    rc = na_tmap_w3d(&tm.w[1], d.scratch, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, C::K(1), C::N(1), Lay::kBK,
                     C::N(1) / Lay::NH / 64);
  if (rc != GP_OK) return rc;
  ChainArgs args;
  std::memset(&args, 0, sizeof(args));
  args.m = m;
  args.num_tiles = static_cast<int>((m + kBM - 1) / kBM);
  args.bias[0] = b0;
  args.bias[1] = b1;
  args.gamma = gamma;
  args.beta = beta;
  args.resid = x;
  args.out = out;
  args.ln_eps = 1e-5f;
  args.status = d.status;
  args.timeout_ns = current_timeout_ns();
  args.inject = current_fault_injection();
  const int grid = args.num_tiles < d.sm_count ? args.num_tiles : d.sm_count;
  {
    // a plain launch (it overlaps no earlier kernel), but its kernel triggers the next launch of
    // the stream early, so the stream's record must not allow early reads after it
    PdlLaunch pdl(stream);
    mlp_stream_kernel<C><<<grid, Lay::kThreads, Lay::kSmemBytes, stream>>>(tm, args);
    PdlIo io;
    io.writes_unknown = true;
    pdl.record(io);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "launch: %s", cudaGetErrorString(e));
  count_launches(2);  // the weight conversion and the chain kernel
  return GP_OK;
}

bool na_aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace

int noalloc_status(bool clear, int* status) {
  int h = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&h, g_noalloc_status, sizeof(int));
  if (e == cudaSuccess && clear && h != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_noalloc_status, &zero, sizeof(int));
  }
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "no-alloc status: %s", cudaGetErrorString(e));
  *status = h;
  return GP_OK;
}

}  // namespace gp

using namespace gp;

extern "C" int gp_gc_edges_bf16_noalloc_out(int64_t m, int act, const void* x, const void* w0,
                                            const void* b0, const void* w1, const void* b1,
                                            const void* gamma, const void* beta, void* out,
                                            void* stream) {
  clear_error();
  if (m < 0) return set_error(GP_ERR_ARG, "m = %lld is negative", (long long)m);
  if (m >= (int64_t(1) << 31)) return set_error(GP_ERR_SHAPE, "m = %lld exceeds 2^31-1", (long long)m);
  if (act != GP_ACT_RELU && act != GP_ACT_SILU)
    return set_error(GP_ERR_UNSUPPORTED, "act %d: only GP_ACT_RELU and GP_ACT_SILU are compiled", act);
  if (x == nullptr || w0 == nullptr || w1 == nullptr || out == nullptr)
    return set_error(GP_ERR_ARG, "x, w0, w1 and out must not be NULL");
  if (!na_aligned(x, 16) || !na_aligned(out, 16) || !na_aligned(w0, 16) || !na_aligned(w1, 16))
    return set_error(GP_ERR_ALIGN, "x, w0, w1 and out must be 16-byte aligned");
  const size_t need = size_t(512) * 512 * 2;  // fp16 copy of w1 [512, 512]
  if (need > kNoAllocScratchBytes)
    return set_error(GP_ERR_SHAPE, "weights need %zu bytes of scratch, the fixed buffer holds %zu",
                     need, kNoAllocScratchBytes);
  if (m == 0) return GP_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(GP_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  NoAllocDevice* d = nullptr;
  int rc = na_setup(dev, &d);
  if (rc != GP_OK) return rc;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (act == GP_ACT_SILU)
    return na_launch<kActSilu>(*d, m, x, w0, b0, w1, b1, gamma, beta, out, s, &d->attr_silu);
  return na_launch<kActRelu>(*d, m, x, w0, b0, w1, b1, gamma, beta, out, s, &d->attr_relu);
}
