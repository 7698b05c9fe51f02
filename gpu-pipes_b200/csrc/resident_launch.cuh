// Host launchers for the weight-resident chain kernel (single CTA and CTA pair).
#pragma once

#include <atomic>
#include <cstring>

#include "chain_registry.h"
#include "mlp_resident.cuh"

namespace gp {

// XM: x mode of mlp_resident_body. 1: c.x = the edge rows ef [m, 128], args.gnodes / gidx set;
// 2: c.x = first source [m, 128], c.x2 = second source [m, K0 - 128].
template <typename T, int K0, int N, int NL, uint32_t ACTS, int TAIL, int NBUF, int CG, int XM = 0>
int launch_resident_cg(const LaunchCtx& c) {
  using L = ResidentLayout<K0, N, NL, NBUF, CG, XM == 1>;
  const void* kern = nullptr;
  if constexpr (CG == 2) {
    kern = reinterpret_cast<const void*>(&mlp_resident_pair_kernel<T, K0, N, NL, ACTS, TAIL, NBUF, XM>);
  } else {
    kern = reinterpret_cast<const void*>(&mlp_resident_kernel<T, K0, N, NL, ACTS, TAIL, NBUF, XM>);
  }
  static unsigned long long done_mask = 0;
  static std::atomic<int> max_clusters[64];
  constexpr int kThr = resident_threads<L, XM>();
  constexpr int kSmem = resident_smem<L, XM>();
  static_assert(kSmem <= kSmemLimit, "shared memory budget");
  int rc = ensure_smem_attr(kern, kSmem, &done_mask);
  if (rc != GP_OK) return rc;
  const int dt = c.spec->dtype;
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  rc = make_tmap_2d(&tm.x, c.x, dt, c.m, XM == 0 ? K0 : 128, kPanel, kBM, 128);
  if (rc == GP_OK && XM == 2) rc = make_tmap_2d(&tm.x2, c.x2, dt, c.m, K0 - 128, kPanel, kBM, 128);
  // x mode 1: the node rows, one row per box for tile::gather4
  if (rc == GP_OK && XM == 1)
    rc = make_tmap_2d(&tm.x2, c.args.gnodes, dt, static_cast<uint64_t>(c.args.n_nodes), 128, kPanel, 1, 128);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out, c.out, dt, c.m, N, 32, 32, 64);
  for (int l = 0; rc == GP_OK && l < NL; ++l)
    rc = make_tmap_2d(&tm.w[l], c.w[l], dt, l == 0 ? K0 : N, N, kPanel, kPanel, 128);
  if (rc != GP_OK) return rc;
  ChainArgs args = c.args;
  args.num_tiles = static_cast<int>((c.m + L::kUnitRows - 1) / L::kUnitRows);
  const uint64_t es = 2, rows = static_cast<uint64_t>(c.m);
  PdlIo io;
  for (int l = 0; l < NL; ++l) {
    io.add(PdlIo::kParam, c.w[l], static_cast<uint64_t>(l == 0 ? K0 : N) * N * es);
    io.add(PdlIo::kParam, args.bias[l], N * es);
  }
  io.add(PdlIo::kParam, args.gamma, N * es);
  io.add(PdlIo::kParam, args.beta, N * es);
  io.add(PdlIo::kX, c.x, rows * (XM == 0 ? K0 : 128) * es);
  if (XM == 2) io.add(PdlIo::kX, c.x2, rows * (K0 - 128) * es);
  if (XM == 1) {
    io.add(PdlIo::kX, args.gnodes, static_cast<uint64_t>(args.n_nodes) * 128 * es);
    io.add(PdlIo::kX, args.gidx[0], rows * 8);
    io.add(PdlIo::kX, args.gidx[1], rows * 8);
  }
  io.add(PdlIo::kWrite, c.out, rows * N * es);
  io.add(PdlIo::kWrite, args.scatter, static_cast<uint64_t>(args.n_nodes) * N * 4);
  PdlLaunch pdl(c.stream);
  args.pdl_early = pdl.early_flags(io);
  if constexpr (CG == 1) {
    const int grid = args.num_tiles < c.sm_count ? args.num_tiles : c.sm_count;
    launch_chain_kernel(&mlp_resident_kernel<T, K0, N, NL, ACTS, TAIL, NBUF, XM>, grid, kThr, kSmem, c.stream, tm, args);
  } else {
    int dev = 0;
    cudaGetDevice(&dev);
    std::atomic<int>& mc_slot = max_clusters[dev & 63];  // filled once per device; racing first calls store the same value
    int mc = mc_slot.load(std::memory_order_relaxed);
    if (mc == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (c.sm_count / 2), 1, 1);
      cfg.blockDim = dim3(kThr, 1, 1);
      cfg.dynamicSmemBytes = kSmem;
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
    launch_chain_kernel(&mlp_resident_pair_kernel<T, K0, N, NL, ACTS, TAIL, NBUF, XM>, 2 * clusters, kThr, kSmem,
                        c.stream, tm, args);
  }
  pdl.record(io);
  return GP_OK;
}

template <typename T, int K0, int N, int NL, uint32_t ACTS, int TAIL, int NBUF = 2>
int launch_resident(const LaunchCtx& c) {
  return launch_resident_cg<T, K0, N, NL, ACTS, TAIL, NBUF, 1>(c);
}

template <typename T, int K0, int N, int NL, uint32_t ACTS, int TAIL, int NBUF = 2>
int launch_resident_pair(const LaunchCtx& c) {
  return launch_resident_cg<T, K0, N, NL, ACTS, TAIL, NBUF, 2>(c);
}

}  // namespace gp
