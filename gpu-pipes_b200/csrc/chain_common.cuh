// Types shared by the fused-chain kernels and the C ABI host code.
#pragma once

#include <cuda.h>  // CUtensorMap (header only; the driver entry point is fetched at run time)
#include <cstdint>

namespace gp {

constexpr int kBM = 128;            // rows per tile: one TMEM lane (and one epilogue thread) per row
constexpr int kPanel = 64;          // 16-bit elements per 128-byte swizzled K panel
constexpr int kPanelBytes = kBM * kPanel * 2;  // one x panel: 128 rows x 128 B = 16 KB
constexpr int kMaxLayers = 12;     // kernels; the public spec (GP_MAX_LAYERS) allows 10
constexpr int kSmemLimit = 232448;  // sm_100 opt-in dynamic shared memory per CTA

// Tail applied after the last GEMM (+bias, +activation) of a chain.
enum Tail : int {
  kTailNone = 0,         // out = act(last GEMM + bias)
  kTailLayerNorm = 1,    // out = LN(last GEMM + bias) * gamma + beta
  kTailResidualLN = 2,   // out = LN(last GEMM + bias + x) * gamma + beta
};

// TMA descriptors for one launch. Passed as a __grid_constant__ kernel parameter.
struct TensorMaps {
  CUtensorMap x;                 // input rows  [M, K0]
  CUtensorMap out;               // output rows [M, N_last]
  CUtensorMap w[kMaxLayers];     // weights [K_l, N_l], row-major (N contiguous)
  CUtensorMap x2;                // second input source (resident kernel, x mode 2)
};

struct ChainArgs {
  int64_t m;                          // rows
  int num_tiles;                      // ceil(m / kBM)
  const void* bias[kMaxLayers];       // [N_l] each (16-bit), may be null (no bias)
  const void* gamma;                  // [N_last] LayerNorm scale
  const void* beta;                   // [N_last] LayerNorm shift
  const void* resid;                  // residual rows [M, N_last] (kTailResidualLN)
  void* out;                          // output rows [M, N_out]
  const void* head_w;                 // narrow head [N_last, HEAD_N] (stream kernel), or null
  const void* head_b;                 // narrow head bias [HEAD_N], or null
  float ln_eps;
  int* status;                        // device status word (0 = ok)
  unsigned long long timeout_ns;      // budget of every bounded wait
  int inject;                         // fault injection: 1 = producer never loads x
  // MeshGraphNet edge update (resident kernel, x mode 1): x = [nodes[gidx[0]] | x | nodes[gidx[1]]]
  const void* gnodes;                 // node rows [n_nodes, 128]
  const int64_t* gidx[2];             // per row: source and destination node
  int64_t n_nodes;
  float* scatter;                     // [n_nodes, N_last] fp32, += out row at gidx[1] (or null)
  void* out2;                         // side output rows [M, N(SIDE)] (stream kernel, SIDE chains)
  int pdl_early;                      // reads allowed before griddepcontrol.wait: 1 parameters, 2 x
};

}  // namespace gp
