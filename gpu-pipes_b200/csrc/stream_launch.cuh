// Host launcher for mlp_stream_kernel.
#pragma once

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

template <class C>
int launch_stream(const LaunchCtx& c) {
  using L = StreamLayout<C>;
  const void* kern = reinterpret_cast<const void*>(&mlp_stream_kernel<C>);
  static unsigned long long done_mask = 0;
  int rc = ensure_smem_attr(kern, L::kSmemBytes, &done_mask);
  if (rc != GP_OK) return rc;
  const int dt = c.spec->dtype;
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  rc = make_tmap_2d(&tm.x, c.x, dt, c.m, C::K(0), kPanel, kBM, 128);
  if (rc == GP_OK && C::TAIL != kTailHead)
    rc = make_tmap_2d(&tm.out, c.out, dt, c.m, C::N(C::NL - 1), 32, 32, 64);
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
    rc = make_tmap_2d(&tm.w[l], wl, conv ? GP_F16 : dt, C::K(l), C::N(l), 64, L::kBK, 128);
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
  const int grid = args.num_tiles < c.sm_count ? args.num_tiles : c.sm_count;
  mlp_stream_kernel<C><<<grid, L::kThreads, L::kSmemBytes, c.stream>>>(tm, args);
  if (scratch != nullptr) workspace_release(c.stream);
  return GP_OK;
}

}  // namespace gp
