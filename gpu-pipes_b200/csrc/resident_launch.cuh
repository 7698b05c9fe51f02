// Host launcher for mlp_resident_kernel.
#pragma once

#include "chain_registry.h"
#include "mlp_resident.cuh"

namespace gp {

template <typename T, int K0, int N, int NL, uint32_t ACTS, int TAIL, int NBUF = 2>
int launch_resident(const LaunchCtx& c) {
  using L = ResidentLayout<K0, N, NL, NBUF>;
  const void* kern = reinterpret_cast<const void*>(&mlp_resident_kernel<T, K0, N, NL, ACTS, TAIL, NBUF>);
  static unsigned long long done_mask = 0;
  int rc = ensure_smem_attr(kern, L::kSmemBytes, &done_mask);
  if (rc != GP_OK) return rc;
  const int dt = c.spec->dtype;
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  rc = make_tmap_2d(&tm.x, c.x, dt, c.m, K0, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out, c.out, dt, c.m, N, 32, 32, 64);
  for (int l = 0; rc == GP_OK && l < NL; ++l)
    rc = make_tmap_2d(&tm.w[l], c.w[l], dt, l == 0 ? K0 : N, N, kPanel, kPanel, 128);
  if (rc != GP_OK) return rc;
  const int grid = c.args.num_tiles < c.sm_count ? c.args.num_tiles : c.sm_count;
  mlp_resident_kernel<T, K0, N, NL, ACTS, TAIL, NBUF><<<grid, L::kThreads, L::kSmemBytes, c.stream>>>(tm, c.args);
  return GP_OK;
}

}  // namespace gp
