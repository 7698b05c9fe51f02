// DLRM feature interaction (graphmodel/dlrm.py:28-42): per sample, F = [bottom-MLP output;
// 26 embedding vectors] (27 x 128), Z = F F^T, and the top MLP's input row
//   out = [bot (128) | Z[a][b] for a > b in row-major order of the strict lower triangle (351) | 0]
// (480 fp16 values; 128 + 351 = 479, padded to 480 like the reference's top MLP input).
//
// Tensor cores on a batched Gram matrix. A 128-row tile holds 4 samples: rows 26 s .. 26 s + 25 are
// sample s's embeddings (the 104 rows are consecutive rows of sparse viewed as [m * 26, 128]),
// rows 104 + s its bottom output (consecutive rows of bot), rows 108..127 zero. K = 128 in two
// SWIZZLE_128B panels, so a tile is 4 TMA requests (2 panels x {104 embedding rows, 4 bottom
// rows}). One M = 128, N = 128, K = 128 MMA of the tile against itself (B = the same K-major tile)
// gives every dot product needed: e_i . e_j of sample s at (26 s + i, 26 s + j), bot . e_i at
// (26 s + i, 104 + s).
//
// Persistent CTAs of 128 threads (three per SM) walk the tiles; the next tile's loads are issued
// into the second buffer while the current one is computed. Thread r (TMEM lane r) handles
// embedding row r: it reads its sample's 26-column window of D (within a 64-column load per warp)
// and the bottom column, and writes its z entries into the sample's output row in shared memory;
// the rows then leave with 16-byte stores.
#include <cuda_fp16.h>

#include <cstdint>

#include "chain_registry.h"
#include "gp_ptx.cuh"

namespace gp {
namespace {

constexpr int kIntThreads = 128;
constexpr int kIntSamples = 4;           // samples per 128-row tile
constexpr int kIntPanel = 16384;         // 128 rows x 128 B
constexpr int kIntTile = 2 * kIntPanel;  // two 64-column panels
constexpr int kIntBufs = 2;
constexpr int kIntOutRow = 960;          // 480 fp16
constexpr int kIntOffOut = kIntBufs * kIntTile;
constexpr int kIntOffBar = kIntOffOut + kIntSamples * kIntOutRow;
constexpr int kIntSmem = kIntOffBar + 64;  // three CTAs per SM (TMEM: 3 x 128 columns)
constexpr uint32_t kIntTx = 2 * (104 + 4) * 128;  // bytes per tile

__global__ void __launch_bounds__(kIntThreads)
    dlrm_interaction_kernel(const __grid_constant__ CUtensorMap tm_e, const __grid_constant__ CUtensorMap tm_b,
                            __half* __restrict__ out, int64_t m, int* status, unsigned long long timeout_ns) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* stage = smem + kIntOffOut;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kIntOffBar);  // [2]
  uint64_t* mma_bar = full + 2;
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + kIntOffBar + 24);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kIntOffBar + 28);
  const int tid = threadIdx.x, warp = tid >> 5;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (tid == 0) atomicCAS(status, 0, kDevBadSmemAlign);
    return;
  }
  // rows 108..127 of every panel stay zero (no load writes them)
  for (int q = tid; q < kIntBufs * 2 * 20 * 8; q += kIntThreads) {
    const int panel = q / 160, rem = q % 160;
    *reinterpret_cast<uint4*>(smem + panel * kIntPanel + (108 + rem / 8) * 128 + (rem % 8) * 16) =
        make_uint4(0, 0, 0, 0);
  }
  if (tid == 0) {
    mbar_init(smem_u32(&full[0]), 1);
    mbar_init(smem_u32(&full[1]), 1);
    mbar_init(smem_u32(mma_bar), 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tm_e);
    prefetch_tmap(&tm_b);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(holder), 128);
    tmem_relinquish();
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *holder;
  const WaitCtx wctx{status, abort_flag, timeout_ns};
  const uint32_t idesc = make_idesc_f16(128, 128, 0, 0, 0);  // fp16, A and B K-major
  const int64_t tiles = (m + kIntSamples - 1) / kIntSamples;
  auto issue = [&](int64_t t, int b) {  // thread 0
    uint8_t* buf = smem + b * kIntTile;
    mbar_arrive_expect_tx(smem_u32(&full[b]), kIntTx);
    for (int p = 0; p < 2; ++p) {
      tma_load_2d(smem_u32(buf + p * kIntPanel), &tm_e, smem_u32(&full[b]), p * 64, static_cast<int>(t * 104));
      tma_load_2d(smem_u32(buf + p * kIntPanel + 104 * 128), &tm_b, smem_u32(&full[b]), p * 64,
                  static_cast<int>(t * 4));
    }
  };
  // this thread's row: sample s, embedding i (rows >= 104 carry no outputs)
  const int s = tid < 104 ? tid / 26 : -1;
  const int i = tid < 104 ? tid % 26 : 0;
  const int c0 = (26 * ((warp * 32) / 26)) < 64 ? 26 * ((warp * 32) / 26) : 64;  // warp's column window
  if (tid == 0 && blockIdx.x < tiles) issue(blockIdx.x, 0);
  uint32_t fph[2] = {0, 0}, mph = 0;
  bool ok = true;
  int k = 0;
#pragma unroll 1
  for (int64_t t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++k) {
    const int b = k & 1;
    // the next tile into the other buffer: freed by the barrier that ended the last iteration
    if (tid == 0 && t + gridDim.x < tiles) issue(t + gridDim.x, b ^ 1);
    if (!mbar_wait(smem_u32(&full[b]), fph[b], wctx, kDevTimeoutProducer)) ok = false;
    fph[b] ^= 1;
    ok = __syncthreads_and(ok) != 0;
    if (!ok) break;
    tc_fence_after();
    const uint8_t* buf = smem + b * kIntTile;
    if (tid == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint64_t d = make_sdesc_sw128(smem_u32(buf) + (kk >> 2) * kIntPanel + (kk & 3) * 32, 16, 1024);
        mma_ss(tmem, d, d, idesc, kk > 0 ? 1u : 0u);
      }
      mma_commit(smem_u32(mma_bar));
    }
    __syncwarp();
    if (!mbar_wait(smem_u32(mma_bar), mph, wctx, kDevTimeoutEpilogue)) ok = false;
    mph ^= 1;
    tc_fence_after();
    uint32_t v[64], vb[32];
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    tmem_ld32(trow + c0, *reinterpret_cast<uint32_t(*)[32]>(v));
    tmem_ld32(trow + c0 + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
    tmem_ld32(trow + 96, vb);
    tmem_wait_ld();
    // bottom rows into the staged output rows: 16 chunks of 16 B per sample, un-swizzled
    if (tid < 64) {
      const int ss = tid >> 4, c = tid & 15;
      const int row = 104 + ss, panel = c >> 3, cp = c & 7;
      *reinterpret_cast<uint4*>(stage + ss * kIntOutRow + c * 16) =
          *reinterpret_cast<const uint4*>(buf + panel * kIntPanel + row * 128 + ((cp ^ (row & 7)) << 4));
    } else if (tid < 68) {
      reinterpret_cast<__half*>(stage + (tid - 64) * kIntOutRow)[479] = __float2half_rn(0.0f);
    }
    if (s >= 0) {
      // z entries of feature a = i + 1 (after the bottom output, feature 0): pairs (a, 0) .. (a, a - 1)
      const int a = i + 1;
      __half* z = reinterpret_cast<__half*>(stage + s * kIntOutRow) + 128 + a * (a - 1) / 2;
      const float bd = __uint_as_float(s == 0 ? vb[8] : s == 1 ? vb[9] : s == 2 ? vb[10] : vb[11]);
      z[0] = __float2half_rn(bd);
      const int j0 = c0 - 26 * s;  // embedding index of window column 0
#pragma unroll
      for (int jj = 0; jj < 64; ++jj) {
        const int j = j0 + jj;
        if (j >= 0 && j < i) z[j + 1] = __float2half_rn(__uint_as_float(v[jj]));
      }
    }
    __syncthreads();
    for (int q = tid; q < kIntSamples * 60; q += kIntThreads) {
      const int ss = q / 60, c = q % 60;
      const int64_t g = t * kIntSamples + ss;
      if (g < m)
        reinterpret_cast<uint4*>(out + g * 480)[c] = *reinterpret_cast<const uint4*>(stage + ss * kIntOutRow + c * 16);
    }
    tc_fence_before();
    // TMEM, the staged rows and this buffer are reused; a wait that ran out ends the loop in every
    // thread at the same point
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
  CUtensorMap tm_e, tm_b;
  rc = make_tmap_2d(&tm_e, sparse, GP_F16, static_cast<uint64_t>(m) * 26, 128, 64, 104, 128);
  if (rc == GP_OK) rc = make_tmap_2d(&tm_b, bot, GP_F16, static_cast<uint64_t>(m), 128, 64, 4, 128);
  if (rc != GP_OK) return rc;
  const int64_t tiles = (m + kIntSamples - 1) / kIntSamples;
  const int64_t want = static_cast<int64_t>(3) * sm_count;
  const int grid = static_cast<int>(tiles < want ? tiles : want);
  dlrm_interaction_kernel<<<grid, kIntThreads, kIntSmem, stream>>>(tm_e, tm_b, static_cast<__half*>(out), m,
                                                                    status, timeout_ns);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GP_OK : set_error(GP_ERR_CUDA, "interaction launch: %s", cudaGetErrorString(e));
}

}  // namespace gp
