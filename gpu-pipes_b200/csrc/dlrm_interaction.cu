// DLRM feature interaction (graphmodel/dlrm.py:28-42): per sample, F = [bottom-MLP output;
// 26 embedding vectors] (27 x 128), Z = F F^T, and the top MLP's input row
//   out = [bot (128) | Z[a][b] for a > b in row-major order of the strict lower triangle (351) | 0]
// (480 fp16 values; 128 + 351 = 479, padded to 480 like the reference's top MLP input).
//
// Tensor cores on a batched Gram matrix: a 128-row tile holds 4 samples x 32 rows (row i < 26:
// embedding i, row 26: the bottom output, rows 27..31: zero), K = 128 in two SWIZZLE_128B panels.
// One M = 128, N = 128, K = 128 MMA of the tile against itself (B = the same K-major tile) gives
// every sample's 27 x 27 Gram matrix in its 32 x 32 diagonal block; the off-diagonal blocks are
// discarded. Warp w of the epilogue holds TMEM lanes 32w..32w+31 -- sample w's rows -- and loads
// its diagonal block (columns 32w..32w+31).
//
// CTAs of 128 threads each take tiles in turn: the 128 threads load a tile (16-byte loads, manual
// SW128 swizzle), thread 0 issues the 8 MMAs, everyone waits for the commit, then reads TMEM and
// writes the rows. Four CTAs per SM (128 TMEM columns each) overlap each other's load latency.
#include <cuda_fp16.h>

#include <cstdint>

#include "chain_registry.h"
#include "gp_ptx.cuh"

namespace gp {
namespace {

constexpr int kIntThreads = 128;
constexpr int kIntSamples = 4;          // samples per 128-row tile
constexpr int kIntTileBytes = 2 * 16384;  // two 64-column panels x 128 rows x 128 B
constexpr int kIntSmem = 56 * 1024;       // sized so that four CTAs fit on an SM (TMEM: 4 x 128 cols)

__global__ void __launch_bounds__(kIntThreads)
    dlrm_interaction_kernel(const __half* __restrict__ bot, const __half* __restrict__ sparse,
                            __half* __restrict__ out, int64_t m, int* status,
                            unsigned long long timeout_ns) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* tile = smem;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + kIntTileBytes);
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + kIntTileBytes + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kIntTileBytes + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) atomicCAS(status, 0, kDevBadSmemAlign);
    return;
  }
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(holder), 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  const WaitCtx wctx{status, abort_flag, timeout_ns};
  const uint32_t idesc = make_idesc_f16(128, 128, 0, 0, 0);  // fp16, A and B K-major
  const int64_t tiles = (m + kIntSamples - 1) / kIntSamples;
  uint32_t phase = 0;
  bool ok = true;
#pragma unroll 1
  for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
    // ---- load the tile: row r = 32 s + i, 16 chunks of 16 B per row; all 16 loads of a thread
    // are issued before any store, so a CTA keeps its whole tile in flight
    {
      uint4 v[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int q = threadIdx.x + u * kIntThreads;
        const int r = q >> 4, c = q & 15;
        const int s = r >> 5, i = r & 31;
        const int64_t g = t * kIntSamples + s;
        v[u] = make_uint4(0, 0, 0, 0);
        if (g < m && i <= 26) {
          const __half* src = i < 26 ? sparse + (g * 26 + i) * 128 : bot + g * 128;
          v[u] = __ldg(reinterpret_cast<const uint4*>(src) + c);
        }
      }
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int q = threadIdx.x + u * kIntThreads;
        const int r = q >> 4, c = q & 15;
        const int panel = c >> 3, cp = c & 7;
        *reinterpret_cast<uint4*>(tile + panel * 16384 + r * 128 + ((cp ^ (r & 7)) * 16)) = v[u];
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint64_t d = make_sdesc_sw128(smem_u32(tile) + (k >> 2) * 16384 + (k & 3) * 32, 16, 1024);
        mma_ss(tmem, d, d, idesc, k > 0 ? 1u : 0u);
      }
      mma_commit(smem_u32(bar));
    }
    __syncwarp();
    if (!mbar_wait(smem_u32(bar), phase, wctx, kDevTimeoutEpilogue)) ok = false;
    phase ^= 1;
    tc_fence_after();
    // ---- epilogue: warp w = sample w of the tile; lane i = row i of its Gram block. The output
    // row (480 halves, 960 B) is assembled in shared memory, then written with 16-byte stores. It
    // goes to bytes [4096 w, 4096 w + 960): sample w's own tile rows 0..7 of the first panel, no
    // longer read by the (complete) MMAs nor by any other warp, and disjoint from its row 26.
    const int64_t g = t * kIntSamples + warp;
    uint32_t v[32];
    tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + warp * 32, v);
    tmem_wait_ld();
    __half* srow = reinterpret_cast<__half*>(tile + warp * 4096);
    if (lane < 16) {  // the bottom output, from its tile row 32 w + 26 (un-swizzled)
      const int r = warp * 32 + 26;
      const int panel = lane >> 3, cp = lane & 7;
      reinterpret_cast<uint4*>(srow)[lane] =
          *reinterpret_cast<const uint4*>(tile + panel * 16384 + r * 128 + ((cp ^ (r & 7)) * 16));
    }
    if (lane < 26) {
      // tile row `lane` is embedding lane = feature a = lane + 1 of F = [bot; e_0 .. e_25]; its
      // pairs (a, b < a) start at a (a - 1) / 2: b = 0 is the bottom output (tile row 26),
      // b = j + 1 is embedding j (tile row j)
      const int a = lane + 1;
      __half* z = srow + 128 + a * (a - 1) / 2;
      z[0] = __float2half_rn(__uint_as_float(v[26]));
      for (int j = 0; j < lane; ++j) z[j + 1] = __float2half_rn(__uint_as_float(v[j]));
    }
    if (lane == 31) srow[479] = __float2half_rn(0.0f);
    __syncwarp();
    if (ok && g < m) {
      const uint4* src = reinterpret_cast<const uint4*>(srow);
      uint4* dst = reinterpret_cast<uint4*>(out + g * 480);
      for (int c = lane; c < 60; c += 32) dst[c] = src[c];
    }
    tc_fence_before();
    // TMEM and the tile are reused by the next tile; a wait that ran out anywhere ends the loop
    // in every thread at the same point
    ok = __syncthreads_and(ok) != 0;
    tc_fence_after();
  }
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace

int launch_dlrm_interaction(int64_t m, const void* bot, const void* sparse, void* out,
                            cudaStream_t stream, int sm_count, int* status,
                            unsigned long long timeout_ns) {
  static unsigned long long done_mask = 0;
  int rc = ensure_smem_attr(reinterpret_cast<const void*>(&dlrm_interaction_kernel), kIntSmem, &done_mask);
  if (rc != GP_OK) return rc;
  const int64_t tiles = (m + kIntSamples - 1) / kIntSamples;
  const int64_t want = static_cast<int64_t>(4) * sm_count;
  const int grid = static_cast<int>(tiles < want ? tiles : want);
  dlrm_interaction_kernel<<<grid, kIntThreads, kIntSmem, stream>>>(
      static_cast<const __half*>(bot), static_cast<const __half*>(sparse), static_cast<__half*>(out), m,
      status, timeout_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GP_OK : set_error(GP_ERR_CUDA, "interaction launch: %s", cudaGetErrorString(e));
}

}  // namespace gp
