// MeshGraphNet message passing around the edge and node MLPs (graphmodel/mgn_dp.py:28-54):
//   edge update  out[e] = LN(MLP([nf[src[e]] | ef[e] | nf[dst[e]]]))      mgn_dp.py:28-32
//   aggregation  agg[v] = sum of out[e] over the edges with dst[e] = v     (UnsortedSegmentSum,
//                                                                          graphmodel/common.py:97-99)
//   node update  out[v] = LN(MLP([nf[v] | agg_0[v] | agg_1[v] ...]))      mgn_dp.py:46-54
// MLP = 128 -> 128 ReLU -> 128 ReLU -> 128 (common/mlps.py MgnMlp), fp16.
//
// The edge update is the weight-resident CTA-pair kernel in x mode 1: the concat is assembled in
// shared memory (node rows gathered by the producer warps, ef by TMA) and never exists in HBM; the
// aggregation is fused into its epilogue (fp32 vector atomics of the stored output rows). The
// node update converts the fp32 aggregates to fp16 once ([n, 128 * n_sets] in the workspace) and
// runs the resident kernel in x mode 2 on [nf | that buffer] through two tensor maps.
#include <cuda_fp16.h>

#include "resident_launch.cuh"

namespace gp {
namespace {
constexpr uint32_t kActsMgn = GP_ACT_RELU | (GP_ACT_RELU << 4);

// dst [n, 128 * n_sets] fp16 = the n_sets fp32 aggregates side by side; 8 values per thread.
__global__ void agg_to_f16_kernel(const float* __restrict__ agg0, const float* __restrict__ agg1,
                                  int n_sets, int64_t n, __half* __restrict__ dst) {
  const int64_t per_row = 16 * n_sets;  // 8-value groups per row
  const int64_t total = n * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / per_row;
    const int g = static_cast<int>(i - row * per_row);
    const int set = g >> 4, c = (g & 15) * 8;
    const float4* src = reinterpret_cast<const float4*>((set == 0 ? agg0 : agg1) + row * 128 + c);
    const float4 a = __ldg(src), b = __ldg(src + 1);
    __half2 h[4] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w),
                    __floats2half2_rn(b.x, b.y), __floats2half2_rn(b.z, b.w)};
    *reinterpret_cast<uint4*>(dst + row * 128 * n_sets + set * 128 + c) = *reinterpret_cast<uint4*>(h);
  }
}
}  // namespace

int launch_mgn_edge_update(const LaunchCtx& base, int64_t m, int64_t n_nodes, const void* nf,
                           const void* ef, const int64_t* srcs, const int64_t* dsts,
                           const void* const* w, const void* const* b, const void* gamma,
                           const void* beta, void* out, float* agg) {
  gp_mlp_spec spec{};
  spec.dtype = GP_F16;
  LaunchCtx c = base;
  c.spec = &spec;
  c.m = m;
  c.x = ef;
  c.out = out;
  c.args.m = m;
  for (int l = 0; l < 3; ++l) {
    c.w[l] = w[l];
    c.args.bias[l] = b != nullptr ? b[l] : nullptr;
  }
  c.args.gamma = gamma;
  c.args.beta = beta;
  c.args.out = out;
  c.args.gnodes = nf;
  c.args.gidx[0] = srcs;
  c.args.gidx[1] = dsts;
  c.args.n_nodes = n_nodes;
  c.args.scatter = agg;
  return launch_resident_cg<__half, 384, 128, 3, kActsMgn, kTailLayerNorm, 2, 2, 1>(c);
}

int launch_mgn_node_update(const LaunchCtx& base, int64_t n, int n_sets, const void* nf,
                           const float* const* aggs, const void* const* w, const void* const* b,
                           const void* gamma, const void* beta, void* out) {
  const size_t h_bytes = static_cast<size_t>(n) * 128 * n_sets * 2;
  void* ws = nullptr;
  int rc = workspace_acquire(h_bytes, base.stream, &ws);
  if (rc != GP_OK) return rc;
  __half* agg16 = static_cast<__half*>(ws);
  {
    const int64_t work = n * 16 * n_sets;
    const int64_t want = (work + 255) / 256;
    const int blocks = static_cast<int>(want < 8 * base.sm_count ? want : 8 * base.sm_count);
    agg_to_f16_kernel<<<blocks, 256, 0, base.stream>>>(aggs[0], n_sets > 1 ? aggs[1] : nullptr, n_sets,
                                                       n, agg16);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    workspace_release(base.stream);
    return set_error(GP_ERR_CUDA, "node aggregate conversion: %s", cudaGetErrorString(e));
  }
  gp_mlp_spec spec{};
  spec.dtype = GP_F16;
  LaunchCtx c = base;
  c.spec = &spec;
  c.m = n;
  c.x = nf;
  c.x2 = agg16;
  c.out = out;
  c.args.m = n;
  for (int l = 0; l < 3; ++l) {
    c.w[l] = w[l];
    c.args.bias[l] = b != nullptr ? b[l] : nullptr;
  }
  c.args.gamma = gamma;
  c.args.beta = beta;
  c.args.out = out;
  rc = n_sets == 1 ? launch_resident_cg<__half, 256, 128, 3, kActsMgn, kTailLayerNorm, 2, 1, 2>(c)
                   : launch_resident_cg<__half, 384, 128, 3, kActsMgn, kTailLayerNorm, 2, 2, 2>(c);
  workspace_release(base.stream);
  return rc;
}

}  // namespace gp
