// Host launcher for mlp_stream_kernel (one CTA per 128-row tile) and mlp_stream_pair_kernel
// (CTA pairs over 256-row units, each CTA staging half of every weight stage).
#pragma once

#include <atomic>
#include <cstring>

#include "chain_registry.h"
#include "mlp_stream.cuh"

namespace gp {

// bf16 -> fp16 copy of a weight matrix (exact for values within the fp16 range).
static __global__ void bf16_to_f16_kernel(const __nv_bfloat16* __restrict__ src, __half* __restrict__ dst,
                                   int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __float2half_rn(__bfloat162float(src[i]));
}

template <class C, int CG = 1>
int launch_stream(const LaunchCtx& c) {
  using L = StreamLayout<C, CG>;
  const void* kern = nullptr;
  if constexpr (CG == 2) {
    kern = reinterpret_cast<const void*>(&mlp_stream_pair_kernel<C>);
  } else {
    kern = reinterpret_cast<const void*>(&mlp_stream_kernel<C>);
  }
  static unsigned long long done_mask = 0;
  static std::atomic<int> max_clusters[64];
  int rc = ensure_smem_attr(kern, L::kSmemBytes, &done_mask);
  if (rc != GP_OK) return rc;
  const int dt = c.spec->dtype;
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  rc = make_tmap_2d(&tm.x, c.x, dt, c.m, C::K(0), kPanel, kBM, 128, c.x_ld);
  if (rc == GP_OK && C::TAIL != kTailHead)
    rc = make_tmap_2d(&tm.out, c.out, dt, c.m, L::kOutN, 32, 32, 64, c.out_ld);
  if constexpr (L::kSkip2 != 0) {
    // second input [m, X2_COLS] as one 64-column panel per tile (columns past X2_COLS read zero)
    if (rc == GP_OK) rc = make_tmap_2d(&tm.x2, c.x2, dt, c.m, C::X2_COLS, kPanel, kBM, 128);
  }
  // fp16 copies of the weights of layers >= 1 (HIDDEN_F16), in the per-device workspace
  void* scratch = nullptr;
  size_t offs[kMaxLayers] = {0};
  if constexpr (C::HIDDEN_F16) {
    size_t total = 0;
    for (int l = 1; l < C::NL; ++l) {
      offs[l] = total;
      total += ((static_cast<size_t>(C::K(l)) * C::N(l) * 2 + 255) / 256) * 256;
    }
    rc = workspace_acquire(total, c.stream, &scratch);
    if (rc != GP_OK) return rc;
    for (int l = 1; l < C::NL; ++l) {
      const int64_t n = static_cast<int64_t>(C::K(l)) * C::N(l);
      bf16_to_f16_kernel<<<static_cast<int>((n + 1023) / 1024), 256, 0, c.stream>>>(
          static_cast<const __nv_bfloat16*>(c.w[l]),
          reinterpret_cast<__half*>(static_cast<char*>(scratch) + offs[l]), n);
    }
  }
  for (int l = 0; rc == GP_OK && l < C::NL; ++l) {
    const bool conv = C::HIDDEN_F16 && l > 0;
    const void* wl = conv ? static_cast<const void*>(static_cast<char*>(scratch) + offs[l]) : c.w[l];
    // one stage = kBK rows of this CTA's columns of one output half
    rc = make_tmap_w3d(&tm.w[l], wl, conv ? GP_F16 : dt, WeightRows<C>::get(l), C::N(l), L::kBK,
                       C::N(l) / L::NH / CG / 64);
  }
  if (rc != GP_OK) {
    if (scratch != nullptr) workspace_release(c.stream);
    return rc;
  }
  ChainArgs args = c.args;
  if constexpr (C::TAIL == kTailHead) {
    args.head_w = c.w[C::NL];
    args.head_b = c.args.bias[C::NL];
  }
  args.num_tiles = static_cast<int>((c.m + kBM * CG - 1) / (kBM * CG));
  const uint64_t es = 2, rows = static_cast<uint64_t>(c.m);
  PdlIo io;
  for (int l = 0; l < C::NL; ++l) {
    const bool conv = C::HIDDEN_F16 && l > 0;
    const void* wl = conv ? static_cast<const void*>(static_cast<char*>(scratch) + offs[l]) : c.w[l];
    io.add(PdlIo::kParam, wl, static_cast<uint64_t>(WeightRows<C>::get(l)) * C::N(l) * es);
    io.add(PdlIo::kParam, args.bias[l], static_cast<uint64_t>(C::N(l)) * es);
  }
  io.add(PdlIo::kParam, args.gamma, static_cast<uint64_t>(C::N(C::NL - 1)) * es);
  io.add(PdlIo::kParam, args.beta, static_cast<uint64_t>(C::N(C::NL - 1)) * es);
  if constexpr (C::TAIL == kTailHead) {
    io.add(PdlIo::kParam, args.head_w, static_cast<uint64_t>(C::N(C::NL - 1)) * C::HEAD_N * es);
    io.add(PdlIo::kParam, args.head_b, static_cast<uint64_t>(C::HEAD_N) * es);
  }
  io.add(PdlIo::kX, c.x, rows * static_cast<uint64_t>(c.x_ld != 0 ? c.x_ld : C::K(0)) * es);
  if constexpr (L::kSkip2 != 0) io.add(PdlIo::kX, c.x2, rows * C::X2_COLS * es);
  io.add(PdlIo::kX, args.resid, rows * C::N(C::NL - 1) * es);
  io.add(PdlIo::kWrite, c.out, rows * static_cast<uint64_t>(c.out_ld != 0 ? c.out_ld : L::kOutN) * es);
  if constexpr (L::kSide > 0) io.add(PdlIo::kWrite, args.out2, rows * C::N(L::kSide) * es);
  PdlLaunch pdl(c.stream);
  args.pdl_early = pdl.early_flags(io);
  if constexpr (CG == 1) {
    const int grid = args.num_tiles < c.sm_count ? args.num_tiles : c.sm_count;
    launch_chain_kernel(&mlp_stream_kernel<C>, grid, L::kThreads, L::kSmemBytes, c.stream, tm, args);
  } else {
    int dev = 0;
    cudaGetDevice(&dev);
    std::atomic<int>& mc_slot = max_clusters[dev & 63];  // filled once per device; racing first calls store the same value
    int mc = mc_slot.load(std::memory_order_relaxed);
    if (mc == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (c.sm_count / 2), 1, 1);
      cfg.blockDim = dim3(L::kThreads, 1, 1);
      cfg.dynamicSmemBytes = L::kSmemBytes;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = 2;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      int n = 0;
      cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
      if (e != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = c.sm_count / 2;
      }
      mc = n;
      mc_slot.store(n, std::memory_order_relaxed);
    }
    const int clusters = args.num_tiles < mc ? args.num_tiles : mc;
    launch_chain_kernel(&mlp_stream_pair_kernel<C>, 2 * clusters, L::kThreads, L::kSmemBytes, c.stream, tm, args);
  }
  pdl.record(io);
  if (scratch != nullptr) workspace_release(c.stream);
  return GP_OK;
}

}  // namespace gp
