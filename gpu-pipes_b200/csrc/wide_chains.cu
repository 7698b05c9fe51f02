// Host orchestration of the chains whose hidden activations are too wide for one SM:
//   BERT-large FFN  ln(x + W2 gelu(W1 x + b1) + b2), 1024 -> 4096 -> 1024, bf16
//                   (apps/bert_ffn/torch/model.py:4-15 at BERT-large widths, GELU(tanh))
//   DLRM top MLP    480 -> 1024 -> 1024 -> 512 -> 256 -> 1, ReLU, sigmoid at the end, fp16
//                   (common/mlps.py:23-35 DlrmMlp([479, 1024, 1024, 512, 256, 1], sigmoid_i=4)),
//                   and the reference app's own widths 512 -> 1024 -> 1024 -> 512 -> 256 -> 64
//                   with ReLU after every layer (apps/dlrm_topmlp/pipelined/val.py:11-12,
//                   DlrmMlp([479 + 33, 1024, 1024, 512, 256, 64]); dlrm_topmlp_pl_ext.cu:34-40)
// Default form: each chain runs over large row chunks whose intermediates live in the per-device
// workspace (measured faster than L2-sized chunks: fewer launches and partial waves, and the HBM
// traffic of the intermediates overlaps the GEMMs); each wide layer is one mlp_gemm_pair_kernel
// launch; the tail (LayerNorm, or the last two DLRM layers with the sigmoid head) is a row kernel
// / the weight-streaming chain kernel. Other form (variant 1): the whole chain as one
// mlp_gemm_chain_kernel launch with its intermediates in rings of row blocks (mlp_gemm_chain.cuh);
// measured slower, see the schedules below.
#include <atomic>
#include <cstdlib>
#include <cstring>

#include "chain_registry.h"
#include "mlp_gemm.cuh"
#include "mlp_gemm_chain.cuh"
#include "stream_launch.cuh"

namespace gp {
namespace {

// CTA-pair launch: 256 x 256 tiles, one cluster of two CTAs per tile in flight.
template <int ACT, bool OUT_F32>
int gemm_launch_t(cudaStream_t s, int sm_count, const TensorMaps& tm, const GemmArgs& g, int a_bf16) {
  using L = GemmLayoutT<2>;
  static unsigned long long done_mask = 0;
  static std::atomic<int> max_clusters[64];
  const void* kern = reinterpret_cast<const void*>(&mlp_gemm_pair_kernel<ACT, OUT_F32>);
  int rc = ensure_smem_attr(kern, L::kSmemBytes, &done_mask);
  if (rc != GP_OK) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& mc_slot = max_clusters[dev & 63];  // filled once per device; racing first calls store the same value
  int mc = mc_slot.load(std::memory_order_relaxed);
  if (mc == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sm_count / 2), 1, 1);
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
      n = sm_count / 2;
    }
    mc = n;
    mc_slot.store(n, std::memory_order_relaxed);
  }
  const int clusters = g.num_tiles < mc ? g.num_tiles : mc;
  {
    // the GEMM reads nothing before its wait; its writes are not listed
    PdlLaunch pdl(s);
    launch_chain_kernel(&mlp_gemm_pair_kernel<ACT, OUT_F32>, 2 * clusters, L::kThreads, L::kSmemBytes, s, tm, g, a_bf16);
    PdlIo io;
    io.writes_unknown = true;
    pdl.record(io);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GP_OK : set_error(GP_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
}

int gemm_launch(cudaStream_t s, int sm_count, const void* a, int a_bf16, int64_t m, int k,
                const void* w, int n, const void* bias, int bias_bf16, const void* resid,
                int resid_bf16, int act, void* out, int out_kind /*0 bf16, 1 f16, 2 f32*/,
                int* status, unsigned long long timeout_ns) {
  if (n % GemmLayout::kBN != 0 || n > GemmLayout::kMaxN)
    return set_error(GP_ERR_UNSUPPORTED, "gemm layer width %d", n);
  TensorMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  const int adt = a_bf16 ? GP_BF16 : GP_F16;
  int rc = make_tmap_2d(&tm.x, a, adt, m, k, kPanel, kBM, 128);
  // each CTA of a pair loads half of the tile's 64-column blocks
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[0], w, adt, k, n, kPanel, GemmLayout::kBN / 64 / 2);
  if (rc == GP_OK) {
    rc = out_kind == 2 ? make_tmap_2d_f32(&tm.out, out, m, n, 32, 32, 128)
                       : make_tmap_2d(&tm.out, out, out_kind == 0 ? GP_BF16 : GP_F16, m, n, 32, 32, 64);
  }
  if (rc != GP_OK) return rc;
  GemmArgs g;
  std::memset(&g, 0, sizeof(g));
  g.m = static_cast<int>(m);
  g.n = n;
  g.k = k;
  g.n_tiles = n / GemmLayout::kBN;
  g.num_tiles = static_cast<int>((m + 2 * kBM - 1) / (2 * kBM)) * g.n_tiles;  // 256-row units
  g.act = act;
  g.out_f32 = out_kind == 2;
  g.out_f16 = out_kind == 1;
  g.bias = bias;
  g.bias_bf16 = bias_bf16;
  g.resid = resid;
  g.resid_bf16 = resid_bf16;
  g.out = out;
  g.status = status;
  g.timeout_ns = timeout_ns;
  const int grid = sm_count;
  const bool f32 = out_kind == 2;
  switch (act) {
    case kActNone: return f32 ? gemm_launch_t<kActNone, true>(s, grid, tm, g, a_bf16)
                              : gemm_launch_t<kActNone, false>(s, grid, tm, g, a_bf16);
    case kActRelu: return f32 ? gemm_launch_t<kActRelu, true>(s, grid, tm, g, a_bf16)
                              : gemm_launch_t<kActRelu, false>(s, grid, tm, g, a_bf16);
    case kActGeluTanh: return f32 ? gemm_launch_t<kActGeluTanh, true>(s, grid, tm, g, a_bf16)
                                  : gemm_launch_t<kActGeluTanh, false>(s, grid, tm, g, a_bf16);
    default: return set_error(GP_ERR_UNSUPPORTED, "gemm activation %d", act);
  }
}

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

// The last two DLRM top layers on the weight-streaming kernel: 512 -> 256 (ReLU) -> 1 (sigmoid).
struct ChainDlrmTail {
  using T = __half;
  static constexpr int NL = 1;
  __host__ __device__ static constexpr int K(int) { return 512; }
  __host__ __device__ static constexpr int N(int) { return 256; }
  __host__ __device__ static constexpr int ACT(int) { return kActRelu; }
  static constexpr int SKIP = 0, TAIL = kTailHead, HEAD_N = 1, HEAD_ACT = kActSigmoid;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 1;
  static constexpr bool SPLIT_ACT = false;
};

// The reference app's tail: 512 -> 256 (ReLU) -> 64 (ReLU), stored as [M, 64].
struct ChainDlrmTailRef {
  using T = __half;
  static constexpr int NL = 2;
  __host__ __device__ static constexpr int K(int l) { return l == 0 ? 512 : 256; }
  __host__ __device__ static constexpr int N(int l) { return l == 0 ? 256 : 64; }
  __host__ __device__ static constexpr int ACT(int) { return kActRelu; }
  static constexpr int SKIP = 0, TAIL = kTailNone, HEAD_N = 0, HEAD_ACT = kActNone;
  static constexpr bool HIDDEN_F16 = false;
  static constexpr int HALVES = 1;
  static constexpr bool SPLIT_ACT = false;
};

// ------------------------------------------------------------------ single-kernel chains
// Schedule of a fused chain: step lag of each layer (layer 0 at 0) and of the LayerNorm tiles, and
// the depth (row blocks) of each layer's output ring. GP_CHAIN_SCHED="l1,l2,...;q" overrides the
// lags of layers 1.. (and the LayerNorm tile, last; non-decreasing) and sets every ring depth
// (measurement only); depths are raised to what keeps every dependency pointing backwards in the
// tile sequence.
struct ChainSched {
  int lag[kChainMaxStages + 1] = {0};
  int ring[kChainMaxStages] = {0};
};

void chain_sched_override(ChainSched* sc, int n_lags) {
  const char* e = std::getenv("GP_CHAIN_SCHED");
  if (e == nullptr || *e == 0) return;
  int v[kChainMaxStages + 1] = {0};
  int n = 0, q = 0;
  const char* p = e;
  while (*p != 0 && *p != ';' && n < n_lags) {
    v[n++] = std::atoi(p);
    while (*p != 0 && *p != ',' && *p != ';') ++p;
    if (*p == ',') ++p;
  }
  if (*p == ';') q = std::atoi(p + 1);
  // lags must not decrease (a layer's tiles of a row block come after the previous layer's in
  // the sequence, the LayerNorm tile after the last layer's); otherwise the override is ignored
  for (int i = 0; i < n; ++i)
    if (v[i] < (i == 0 ? 0 : v[i - 1])) return;
  for (int i = 0; i < n; ++i) sc->lag[i + 1] = v[i];
  if (q > 0)
    for (int s = 0; s < kChainMaxStages; ++s) sc->ring[s] = q;
}

int chain_launch(cudaStream_t s, int sm_count, const GemmChainMaps& tm, const GemmChainArgs& g) {
  using L = GemmChainLayout;
  static unsigned long long done_mask = 0;
  static std::atomic<int> max_clusters[64];
  const void* kern = reinterpret_cast<const void*>(&mlp_gemm_chain_kernel);
  int rc = ensure_smem_attr(kern, L::kSmemBytes, &done_mask);
  if (rc != GP_OK) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  std::atomic<int>& mc_slot = max_clusters[dev & 63];  // filled once per device; racing first calls store the same value
  int mc = mc_slot.load(std::memory_order_relaxed);
  if (mc == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (sm_count / 2), 1, 1);
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
      n = sm_count / 2;
    }
    mc = n;
    mc_slot.store(n, std::memory_order_relaxed);
  }
  // at most the co-resident clusters; a pair that is not resident claims no tile, so no tile waits on it
  const int clusters = g.total < mc ? g.total : mc;
  {
    PdlLaunch pdl(s);
    launch_chain_kernel(&mlp_gemm_chain_kernel, 2 * clusters, L::kThreads, L::kSmemBytes, s, tm, g);
    PdlIo io;
    io.writes_unknown = true;
    pdl.record(io);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? GP_OK : set_error(GP_ERR_CUDA, "chain launch: %s", cudaGetErrorString(e));
}

// Fills the schedule fields of g from sc (n_stages layers, optional LayerNorm tiles) and sizes the
// rings: a ring of q row blocks is overwritten by the row block q later, which must come after
// that ring's consumers in the sequence (q > consumer lag - producer lag).
void chain_schedule(GemmChainArgs* g, ChainSched sc, int ln) {
  const int nb = g->n_blocks;
  g->total = 0;
  for (int s = 0; s < g->n_stages; ++s) {
    g->st[s].lag = sc.lag[s];
    g->total += nb * g->st[s].n_tiles;
  }
  g->ln = ln;
  g->ln_lag = ln ? sc.lag[g->n_stages] : 0;
  if (ln) g->total += nb;
  int last = g->ln_lag;
  for (int s = 0; s < g->n_stages; ++s) last = sc.lag[s] > last ? sc.lag[s] : last;
  g->n_steps = last + nb;
  for (int s = 0; s < g->n_stages; ++s) {
    const bool consumed = s + 1 < g->n_stages || ln;
    if (!consumed) {
      g->st[s].ring_q = 0;
      continue;
    }
    const int next_lag = s + 1 < g->n_stages ? sc.lag[s + 1] : g->ln_lag;
    int q = sc.ring[s];
    if (q < next_lag - sc.lag[s] + 1) q = next_lag - sc.lag[s] + 1;
    if (q > nb) q = nb;
    g->st[s].ring_q = q;
  }
}

}  // namespace

// BERT-large FFN (bf16): hidden activations kept in fp16 (as the other bf16 chains), the second
// GEMM on an fp16 copy of W2, pre-LayerNorm rows in fp32.
int launch_bert_ffn_bf16(const LaunchCtx& c) {
  constexpr int H = 1024, F = 4096;
  // 16,384-row chunks: h (128 MB) and y (64 MB) overflow L2, but the extra HBM traffic overlaps
  // the GEMMs, and fewer, larger launches lose less to partial last waves (measured 0.348 ms with
  // 4,096-row chunks, 0.279 with 9,472, 0.253 with 16,384).
  constexpr int64_t kChunk = 16384;
  const int64_t chunk = c.m < kChunk ? c.m : kChunk;
  const size_t w2_bytes = align256(size_t(F) * H * 2);
  const size_t h_bytes = align256(size_t(chunk) * F * 2);
  const size_t y_bytes = align256(size_t(chunk) * H * 4);
  void* ws = nullptr;
  int rc = workspace_acquire(w2_bytes + h_bytes + y_bytes, c.stream, &ws);
  if (rc != GP_OK) return rc;
  char* base = static_cast<char*>(ws);
  void* w2h = base;
  void* h = base + w2_bytes;
  float* y = reinterpret_cast<float*>(base + w2_bytes + h_bytes);
  const int64_t nw = int64_t(F) * H;
  bf16_to_f16_kernel<<<static_cast<int>((nw + 1023) / 1024), 256, 0, c.stream>>>(
      static_cast<const __nv_bfloat16*>(c.w[1]), static_cast<__half*>(w2h), nw);
  const int* st = c.args.status;
  for (int64_t r0 = 0; rc == GP_OK && r0 < c.m; r0 += chunk) {
    const int64_t rows = (c.m - r0) < chunk ? (c.m - r0) : chunk;
    const void* xr = static_cast<const char*>(c.x) + r0 * H * 2;
    rc = gemm_launch(c.stream, c.sm_count, xr, 1, rows, H, c.w[0], F, c.args.bias[0], 1, nullptr, 0,
                     kActGeluTanh, h, 1, const_cast<int*>(st), c.args.timeout_ns);
    if (rc == GP_OK)
      rc = gemm_launch(c.stream, c.sm_count, h, 0, rows, F, w2h, H, c.args.bias[1], 1, xr, 1,
                       kActNone, y, 2, const_cast<int*>(st), c.args.timeout_ns);
    if (rc == GP_OK) {
      row_layernorm_kernel<H><<<static_cast<int>((rows + 7) / 8), 256, 0, c.stream>>>(
          y, c.args.gamma, c.args.beta, 1, c.args.ln_eps, rows,
          static_cast<char*>(c.out) + r0 * H * 2, 1);
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) rc = set_error(GP_ERR_CUDA, "layernorm launch: %s", cudaGetErrorString(e));
    }
  }
  workspace_release(c.stream);
  return rc;
}

// DLRM top MLP (fp16): three wide layers on mlp_gemm_kernel, then the last two layers (512 -> 256
// -> 1 sigmoid head, or 512 -> 256 -> 64) on the streaming chain kernel. The tail runs once per two
// row chunks (h3 holds both), so each of its launches has two 128-row tiles per SM to pipeline
// instead of one.
template <class Tail>
int launch_dlrm_top_t(const LaunchCtx& c) {
  const int n_out = c.spec->widths[5];
  // Chunks of up to 262,144 rows: the intermediates (h1 + h2 + 2 x h3 = 1.5 GB at full size) go
  // through HBM, but the traffic overlaps the GEMMs and large launches lose little to partial
  // last waves. Measured at M = 262,144: 1.44 ms with 16,384-row (L2-sized) chunks, 1.28 with
  // 18,944 (whole waves), 1.05 with 75,776, 0.98 with one chunk.
  constexpr int64_t kChunk = 262144;
  const int64_t chunk = c.m < kChunk ? c.m : kChunk;
  const size_t h1_bytes = align256(size_t(chunk) * 1024 * 2);
  const size_t h3_bytes = align256(size_t(2 * chunk) * 512 * 2);
  void* ws = nullptr;
  int rc = workspace_acquire(2 * h1_bytes + h3_bytes, c.stream, &ws);
  if (rc != GP_OK) return rc;
  char* base = static_cast<char*>(ws);
  void* h1 = base;
  void* h2 = base + h1_bytes;
  char* h3 = base + 2 * h1_bytes;
  int* st = c.args.status;
  const int k0 = c.spec->widths[0];
  for (int64_t r0 = 0; rc == GP_OK && r0 < c.m; r0 += 2 * chunk) {
    int64_t tail_rows = 0;
    for (int sub = 0; rc == GP_OK && sub < 2; ++sub) {
      const int64_t s0 = r0 + sub * chunk;
      if (s0 >= c.m) break;
      const int64_t rows = (c.m - s0) < chunk ? (c.m - s0) : chunk;
      const void* xr = static_cast<const char*>(c.x) + s0 * k0 * 2;
      void* h3s = h3 + tail_rows * 512 * 2;
      rc = gemm_launch(c.stream, c.sm_count, xr, 0, rows, k0, c.w[0], 1024, c.args.bias[0], 0, nullptr,
                       0, kActRelu, h1, 1, st, c.args.timeout_ns);
      if (rc == GP_OK)
        rc = gemm_launch(c.stream, c.sm_count, h1, 0, rows, 1024, c.w[1], 1024, c.args.bias[1], 0,
                         nullptr, 0, kActRelu, h2, 1, st, c.args.timeout_ns);
      if (rc == GP_OK)
        rc = gemm_launch(c.stream, c.sm_count, h2, 0, rows, 1024, c.w[2], 512, c.args.bias[2], 0,
                         nullptr, 0, kActRelu, h3s, 1, st, c.args.timeout_ns);
      tail_rows += rows;
    }
    if (rc == GP_OK) {
      gp_mlp_spec tail_spec = *c.spec;
      LaunchCtx t = c;
      t.spec = &tail_spec;
      t.m = tail_rows;
      t.x = h3;
      t.out = static_cast<char*>(c.out) + r0 * n_out * 2;
      t.w[0] = c.w[3];
      t.w[1] = c.w[4];
      t.args.bias[0] = c.args.bias[3];
      t.args.bias[1] = c.args.bias[4];
      t.args.m = tail_rows;
      t.args.num_tiles = static_cast<int>((tail_rows + kBM - 1) / kBM);
      t.args.out = t.out;
      rc = launch_stream<Tail>(t);
    }
  }
  workspace_release(c.stream);
  return rc;
}

// ------------------------------------------------------------------ single-kernel forms
namespace {

ChainStageArgs chain_stage(int n, int k, int act, int out_kind, int a_bf16, int out_bf16, int bias_off,
                           const void* bias, int bias_bf16, const void* resid, int resid_bf16) {
  ChainStageArgs st;
  std::memset(&st, 0, sizeof(st));
  st.n = n;
  st.k = k;
  st.n_tiles = n / GemmChainLayout::kBN;
  st.act = act;
  st.out_kind = out_kind;
  st.a_bf16 = a_bf16;
  st.out_bf16 = out_bf16;
  st.bias_off = bias_off;
  st.bias = bias;
  st.bias_bf16 = bias_bf16;
  st.resid = resid;
  st.resid_bf16 = resid_bf16;
  return st;
}

size_t ring_bytes(int q, int n, int elem) { return align256(size_t(q) * 256 * n * elem); }

}  // namespace

// BERT-large FFN as one kernel: layer 0 (1024 -> 4096, GELU) into an fp16 ring, layer 1 (4096 ->
// 1024, + x) into an fp32 ring, LayerNorm tiles into out. W2 is used as an fp16 copy (the hidden
// activations are fp16, as on the layer-by-layer path).
int launch_bert_ffn_bf16_chain(const LaunchCtx& c) {
  constexpr int H = 1024, F = 4096;
  GemmChainArgs g;
  std::memset(&g, 0, sizeof(g));
  g.m = static_cast<int>(c.m);
  g.n_blocks = static_cast<int>((c.m + 255) / 256);
  g.n_stages = 2;
  g.st[0] = chain_stage(F, H, kActGeluTanh, 0, 1, 0, 0, c.args.bias[0], 1, nullptr, 0);
  g.st[1] = chain_stage(H, F, kActNone, 1, 0, 0, F, c.args.bias[1], 1, c.x, 1);
  ChainSched sc;
  // measured best of the schedules tried (0.342-0.345 ms at M = 16,384; shorter lags stall on
  // dependencies, e.g. 0.44 ms at 8 / 20 with 16-block rings)
  sc.lag[1] = 16;
  sc.lag[2] = 40;
  sc.ring[0] = 40;
  sc.ring[1] = 40;
  chain_sched_override(&sc, 2);
  chain_schedule(&g, sc, 1);
  const int nb = g.n_blocks;
  const size_t w2_bytes = align256(size_t(F) * H * 2);
  const size_t h_bytes = ring_bytes(g.st[0].ring_q, F, 2);
  const size_t y_bytes = ring_bytes(g.st[1].ring_q, H, 4);
  const size_t cnt_ints = size_t(3) * nb + 1;  // completion counters, then the claim counter
  const size_t cnt_bytes = align256(cnt_ints * sizeof(int));
  void* ws = nullptr;
  int rc = workspace_acquire(w2_bytes + h_bytes + y_bytes + cnt_bytes, c.stream, &ws);
  if (rc != GP_OK) return rc;
  char* base = static_cast<char*>(ws);
  void* w2h = base;
  void* hring = base + w2_bytes;
  void* yring = base + w2_bytes + h_bytes;
  int* counters = reinterpret_cast<int*>(base + w2_bytes + h_bytes + y_bytes);
  const int64_t nw = int64_t(F) * H;
  bf16_to_f16_kernel<<<static_cast<int>((nw + 1023) / 1024), 256, 0, c.stream>>>(
      static_cast<const __nv_bfloat16*>(c.w[1]), static_cast<__half*>(w2h), nw);
  cudaError_t e = cudaMemsetAsync(counters, 0, cnt_ints * sizeof(int), c.stream);
  if (e != cudaSuccess) rc = set_error(GP_ERR_CUDA, "counter reset: %s", cudaGetErrorString(e));
  GemmChainMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  const uint64_t hq = uint64_t(g.st[0].ring_q) * 256, yq = uint64_t(g.st[1].ring_q) * 256;
  if (rc == GP_OK) rc = make_tmap_2d(&tm.a[0], c.x, GP_BF16, c.m, H, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[0], c.w[0], GP_BF16, H, F, kPanel, 2);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out[0], hring, GP_F16, hq, F, 32, 32, 64);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.a[1], hring, GP_F16, hq, F, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[1], w2h, GP_F16, F, H, kPanel, 2);
  if (rc == GP_OK) rc = make_tmap_2d_f32(&tm.out[1], yring, yq, H, 32, 32, 128);
  if (rc == GP_OK) {
    g.counters = counters;
    g.next_tile = counters + cnt_ints - 1;
    g.ln_n = H;
    g.ln_ring = static_cast<const float*>(yring);
    g.gamma = c.args.gamma;
    g.beta = c.args.beta;
    g.g_bf16 = 1;
    g.ln_eps = c.args.ln_eps;
    g.out = c.out;
    g.out_bf16 = 1;
    g.bias_total = F + H;
    g.status = c.args.status;
    g.timeout_ns = c.args.timeout_ns;
    g.inject = c.args.inject;
    rc = chain_launch(c.stream, c.sm_count, tm, g);
  }
  workspace_release(c.stream);
  return rc;
}

// DLRM top MLP as one kernel: three wide layers through fp16 rings, then 512 -> 256 (ReLU) with
// the 256 -> 1 sigmoid head in its epilogue.
int launch_dlrm_top_f16_chain(const LaunchCtx& c) {
  const int k0 = c.spec->widths[0];
  GemmChainArgs g;
  std::memset(&g, 0, sizeof(g));
  g.m = static_cast<int>(c.m);
  g.n_blocks = static_cast<int>((c.m + 255) / 256);
  g.n_stages = 4;
  g.st[0] = chain_stage(1024, k0, kActRelu, 0, 0, 0, 0, c.args.bias[0], 0, nullptr, 0);
  g.st[1] = chain_stage(1024, 1024, kActRelu, 0, 0, 0, 1024, c.args.bias[1], 0, nullptr, 0);
  g.st[2] = chain_stage(512, 1024, kActRelu, 0, 0, 0, 2048, c.args.bias[2], 0, nullptr, 0);
  g.st[3] = chain_stage(256, 512, kActRelu, 2, 0, 0, 2560, c.args.bias[3], 0, nullptr, 0);
  ChainSched sc;
  // measured best of the schedules tried (1.25 ms at M = 262,144; 6 / 20 / 32 with 24-block rings
  // stalled on dependencies at 2.4 ms)
  sc.lag[1] = 20;
  sc.lag[2] = 60;
  sc.lag[3] = 100;
  sc.ring[0] = sc.ring[1] = sc.ring[2] = 120;
  chain_sched_override(&sc, 3);
  chain_schedule(&g, sc, 0);
  const int nb = g.n_blocks;
  const size_t r0 = ring_bytes(g.st[0].ring_q, 1024, 2), r1 = ring_bytes(g.st[1].ring_q, 1024, 2);
  const size_t r2 = ring_bytes(g.st[2].ring_q, 512, 2);
  const size_t cnt_ints = size_t(5) * nb + 1;  // completion counters, then the claim counter
  const size_t cnt_bytes = align256(cnt_ints * sizeof(int));
  void* ws = nullptr;
  int rc = workspace_acquire(r0 + r1 + r2 + cnt_bytes, c.stream, &ws);
  if (rc != GP_OK) return rc;
  char* base = static_cast<char*>(ws);
  void* h1 = base;
  void* h2 = base + r0;
  void* h3 = base + r0 + r1;
  int* counters = reinterpret_cast<int*>(base + r0 + r1 + r2);
  cudaError_t e = cudaMemsetAsync(counters, 0, cnt_ints * sizeof(int), c.stream);
  if (e != cudaSuccess) rc = set_error(GP_ERR_CUDA, "counter reset: %s", cudaGetErrorString(e));
  GemmChainMaps tm;
  std::memset(&tm, 0, sizeof(tm));
  const uint64_t q0 = uint64_t(g.st[0].ring_q) * 256, q1 = uint64_t(g.st[1].ring_q) * 256;
  const uint64_t q2 = uint64_t(g.st[2].ring_q) * 256;
  if (rc == GP_OK) rc = make_tmap_2d(&tm.a[0], c.x, GP_F16, c.m, k0, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[0], c.w[0], GP_F16, k0, 1024, kPanel, 2);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out[0], h1, GP_F16, q0, 1024, 32, 32, 64);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.a[1], h1, GP_F16, q0, 1024, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[1], c.w[1], GP_F16, 1024, 1024, kPanel, 2);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out[1], h2, GP_F16, q1, 1024, 32, 32, 64);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.a[2], h2, GP_F16, q1, 1024, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[2], c.w[2], GP_F16, 1024, 512, kPanel, 2);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.out[2], h3, GP_F16, q2, 512, 32, 32, 64);
  if (rc == GP_OK) rc = make_tmap_2d(&tm.a[3], h3, GP_F16, q2, 512, kPanel, kBM, 128);
  if (rc == GP_OK) rc = make_tmap_w3d(&tm.w[3], c.w[3], GP_F16, 512, 256, kPanel, 2);
  if (rc == GP_OK) {
    tm.out[3] = tm.out[2];  // the head layer stores no rows through a map
    g.counters = counters;
    g.next_tile = counters + cnt_ints - 1;
    g.out = c.out;
    g.out_bf16 = 0;
    g.head_w = c.w[4];
    g.head_b = c.args.bias[4];
    g.bias_total = 2816;
    g.status = c.args.status;
    g.timeout_ns = c.args.timeout_ns;
    g.inject = c.args.inject;
    rc = chain_launch(c.stream, c.sm_count, tm, g);
  }
  workspace_release(c.stream);
  return rc;
}

int launch_dlrm_top_f16(const LaunchCtx& c) { return launch_dlrm_top_t<ChainDlrmTail>(c); }
int launch_dlrm_top_f16_ref(const LaunchCtx& c) { return launch_dlrm_top_t<ChainDlrmTailRef>(c); }

}  // namespace gp
