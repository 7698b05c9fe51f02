// Instantiations and host launcher of the TMEM-activation chain kernel (mlp_tmem.cuh).
#include <atomic>
#include <cstring>
#include <type_traits>

#include "chain_registry.h"
#include "mlp_tmem.cuh"
#include "stream_launch.cuh"

namespace gp {
namespace {

// DLRM bottom MLP (common/mlps.py:23-35 DlrmMlp([K0, 512, 256, 128])), ReLU after every layer.
template <int K0_>
struct TmemDlrmBot {
  using T = __half;
  static constexpr int NL = 3;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? K0_ : (l == 1 ? 512 : 256); }
  __host__ __device__ static constexpr int N(int l) { return l == 0 ? 512 : (l == 1 ? 256 : 128); }
  __host__ __device__ static constexpr int ACT(int) { return kActRelu; }
  static constexpr int TAIL = kTailNone;
  static constexpr bool HIDDEN_F16 = false;
};

// The reference's BERT FFN (apps/bert_ffn/torch/model.py:4-15; H = 128, ff = 512): ReLU, then
// + x and LayerNorm. bf16 data keeps the hidden activation in fp16.
template <typename TT>
struct TmemFfnResLn {
  using T = TT;
  static constexpr int NL = 2;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? 128 : 512; }
  __host__ __device__ static constexpr int N(int l) { return l == 0 ? 512 : 128; }
  __host__ __device__ static constexpr int ACT(int l) { return l == 0 ? kActRelu : kActNone; }
  static constexpr int TAIL = kTailResidualLN;
  static constexpr bool HIDDEN_F16 = std::is_same<TT, __nv_bfloat16>::value;
};

template <class C, int CG = 1>
int launch_tmem(const LaunchCtx& c) {
  using L = TmemLayout<C, CG>;
  const void* kern = CG == 2 ? reinterpret_cast<const void*>(&mlp_tmem_pair_kernel<C>)
                             : reinterpret_cast<const void*>(&mlp_tmem_kernel<C>);
  static unsigned long long done_mask = 0;
  static std::atomic<int> max_clusters[64];
  int rc = ensure_smem_attr(kern, L::kSmemBytes, &done_mask);
  if (rc != GP_OK) return rc;
  const int dt = c.spec->dtype;
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  rc = make_tmap_2d(&tm.x, c.x, dt, c.m, C::K(0), kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out, c.out, dt, c.m, L::NLast, 32, 32, 64);
  // fp16 copies of the weights of layers >= 1 (bf16 data with fp16 hidden activations)
  void* scratch = nullptr;
  size_t offs[kMaxLayers] = {0};
  if constexpr (C::HIDDEN_F16) {
    size_t total = 0;
    for (int l = 1; l < C::NL; ++l) {
      offs[l] = total;
      total += ((static_cast<size_t>(C::K(l)) * C::N(l) * 2 + 255) / 256) * 256;
    }
    if (rc == GP_OK) rc = workspace_acquire(total, c.stream, &scratch);
    if (rc != GP_OK) return rc;
    for (int l = 1; l < C::NL; ++l) {
      const int64_t n = static_cast<int64_t>(C::K(l)) * C::N(l);
      bf16_to_f16_kernel<<<static_cast<int>((n + 1023) / 1024), 256, 0, c.stream>>>(
          static_cast<const __nv_bfloat16*>(c.w[l]),
          reinterpret_cast<__half*>(static_cast<char*>(scratch) + offs[l]), n);
    }
  }
  // first layer: stages of kBK0 rows x one 128-column chunk (two 64-column blocks, one per CTA
  // of a pair); later layers: stages of kBK rows x all N columns (half per CTA of a pair)
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[0], c.w[0], dt, C::K(0), C::N(0), L::kBK0, 2 / CG);
  for (int l = 1; rc == GP_OK && l < C::NL; ++l) {
    const void* wl = C::HIDDEN_F16 ? static_cast<const void*>(static_cast<char*>(scratch) + offs[l]) : c.w[l];
    rc = make_tmap_w3d(&tm.w[l], wl, C::HIDDEN_F16 ? GP_F16 : dt, C::K(l), C::N(l), L::kBK, C::N(l) / 64 / CG);
  }
  if (rc != GP_OK) {
    if (scratch != nullptr) workspace_release(c.stream);
    return rc;
  }
  ChainArgs args = c.args;
  args.num_tiles = static_cast<int>((c.m + L::kUnitRows - 1) / L::kUnitRows);
  const uint64_t es = 2, rows = static_cast<uint64_t>(c.m);
  PdlIo io;
  for (int l = 0; l < C::NL; ++l) {
    const void* wl = (C::HIDDEN_F16 && l > 0) ? static_cast<const void*>(static_cast<char*>(scratch) + offs[l]) : c.w[l];
    io.add(PdlIo::kParam, wl, static_cast<uint64_t>(C::K(l)) * C::N(l) * es);
    io.add(PdlIo::kParam, args.bias[l], static_cast<uint64_t>(C::N(l)) * es);
  }
  io.add(PdlIo::kParam, args.gamma, static_cast<uint64_t>(L::NLast) * es);
  io.add(PdlIo::kParam, args.beta, static_cast<uint64_t>(L::NLast) * es);
  io.add(PdlIo::kX, c.x, rows * C::K(0) * es);
  io.add(PdlIo::kWrite, c.out, rows * L::NLast * es);
  PdlLaunch pdl(c.stream);
  args.pdl_early = pdl.early_flags(io);
  if constexpr (CG == 1) {
    const int grid = args.num_tiles < c.sm_count ? args.num_tiles : c.sm_count;
    launch_chain_kernel(&mlp_tmem_kernel<C>, grid, L::kThreads, L::kSmemBytes, c.stream, tm, args);
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
    launch_chain_kernel(&mlp_tmem_pair_kernel<C>, 2 * clusters, L::kThreads, L::kSmemBytes, c.stream, tm, args);
  }
  pdl.record(io);
  if (scratch != nullptr) workspace_release(c.stream);
  return GP_OK;
}

}  // namespace

int launch_dlrm_bot_f16_tmem(const LaunchCtx& c) { return launch_tmem<TmemDlrmBot<16>>(c); }
int launch_dlrm_bot_f16_k32_tmem(const LaunchCtx& c) { return launch_tmem<TmemDlrmBot<32>>(c); }
int launch_dlrm_bot_f16_tmem_pair(const LaunchCtx& c) { return launch_tmem<TmemDlrmBot<16>, 2>(c); }
int launch_dlrm_bot_f16_k32_tmem_pair(const LaunchCtx& c) { return launch_tmem<TmemDlrmBot<32>, 2>(c); }

// The residual of this kernel is x itself (read from the resident x tile); a chain whose residual
// rows are another tensor (the attention-output block's first stage) runs on the streaming kernel.
int launch_ffn_resln_f16_h128(const LaunchCtx& c);
int launch_ffn_resln_bf16_h128(const LaunchCtx& c);
int launch_ffn_resln_f16_h128_tmem(const LaunchCtx& c) {
  if (c.args.resid != c.x) return launch_ffn_resln_f16_h128(c);
  return launch_tmem<TmemFfnResLn<__half>>(c);
}
int launch_ffn_resln_bf16_h128_tmem(const LaunchCtx& c) {
  if (c.args.resid != c.x) return launch_ffn_resln_bf16_h128(c);
  return launch_tmem<TmemFfnResLn<__nv_bfloat16>>(c);
}
int launch_ffn_resln_f16_h128_tmem_pair(const LaunchCtx& c) {
  if (c.args.resid != c.x) return launch_ffn_resln_f16_h128(c);
  return launch_tmem<TmemFfnResLn<__half>, 2>(c);
}
int launch_ffn_resln_bf16_h128_tmem_pair(const LaunchCtx& c) {
  if (c.args.resid != c.x) return launch_ffn_resln_bf16_h128(c);
  return launch_tmem<TmemFfnResLn<__nv_bfloat16>, 2>(c);
}

}  // namespace gp
